"""Sampled parity checks at full workload sizes -- TEST INFRASTRUCTURE ONLY.

The per-document MaxSim math does not depend on which other documents share
a launch, so a launch over a whole configuration (100000 documents, every
persistent CTA looping over many work items) is checked on a seeded sample
of its documents against the CPU oracle (oracle/maxsim_oracle.py, pinned to
the reference's golden vectors). Used by the GPU tests and by bench.py after
its timed region; never by the product.

Every function takes numpy arrays and returns a dict with `checked` (the
number of query-document scores or gradient rows compared), `max_abs_err`
and `ok`; nothing raises, so a benchmark can report the result.
Tolerance: abs 1e-2 + rel 1e-3 (the north star's bar for scores and
gradients).
"""
from __future__ import annotations

import numpy as np

from . import maxsim_oracle as O

ATOL, RTOL = 1e-2, 1e-3


def sample_docs(B: int, n: int, seed: int = 0) -> np.ndarray:
    """A sorted seeded sample of min(n, B) distinct document indices, plus
    the first and the last document."""
    rng = np.random.default_rng(seed)
    n = min(n, B)
    idx = set(rng.choice(B, size=n, replace=False).tolist())
    idx.update({0, B - 1})
    return np.array(sorted(idx), dtype=np.int64)


def _compare(got, want, what: str) -> dict:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    if got.shape != want.shape:
        return {"checked": 0, "max_abs_err": None, "ok": False, "what": f"{what}: shape {got.shape} != {want.shape}"}
    ninf = np.isneginf(want)
    same_inf = bool(np.array_equal(np.isneginf(got), ninf))
    fin = ~ninf
    err = np.abs(got[fin] - want[fin])
    bound = ATOL + RTOL * np.abs(want[fin])
    ok = same_inf and bool(np.all(err <= bound)) and bool(np.all(np.isfinite(got[fin])))
    return {"checked": int(want.size), "max_abs_err": float(err.max()) if err.size else 0.0, "ok": ok}


def check_scores(Q, D_rows, got, lens_rows=None) -> dict:
    """Scores of sampled documents. Q: [Nq, Lq, d]; D_rows: [n, Ld, d] (the
    sampled documents); got: [Nq, n] GPU scores of those documents."""
    want = O.maxsim_batched(Q, D_rows, lens_rows)
    return _compare(got, want, "scores")


def check_int8(Q, u8_rows, sc_rows, mn_rows, got, lens_rows=None) -> dict:
    """INT8 scores of sampled documents against maxsim_naive on the
    dequantised documents. Q: [Lq, d]; got: [n]."""
    want = O.maxsim(Q, O.dequantize_int8(u8_rows, sc_rows, mn_rows), lens_rows)
    return _compare(got, want, "int8 scores")


def check_fp8(Q, codes_f32_rows, sc_rows, got, lens_rows=None) -> dict:
    """FP8 scores of sampled documents against maxsim_naive on the
    dequantised documents (e4m3 value * per-token scale). Q: [Lq, d]; got: [n]."""
    want = O.maxsim(Q, O.dequantize_fp8(codes_f32_rows, sc_rows), lens_rows)
    return _compare(got, want, "fp8 scores")


def check_train(Q, D_rows, lens_rows, g_rows, scores_rows, am_rows, dD_rows,
                dq_rows_idx, dq_got, dq_want_inputs, eps: float = 1e-4) -> dict:
    """Training forward + backward on sampled documents, tie-aware.

    Q: [Nq, Lq, d]; D_rows [n, Ld, d], lens_rows [n], g_rows [Nq, n] the
    upstream gradient of those documents; scores_rows [Nq, n] and
    am_rows [Nq, n, Lq] the GPU forward (scores, argmax); dD_rows [n, Ld, d]
    the GPU dD of those documents.
    1. scores match the oracle;
    2. the GPU argmax is an eps-argmax of each row (ties may go either way
       under a different summation order), -1 exactly for empty documents;
    3. dD of the sampled documents equals the closed form for the GPU argmax;
    4. dQ rows: dq_rows_idx [(n, q)], dq_got [r, d] the GPU rows and
       dq_want_inputs = (g_all [Nq, B], Dsel [r, B, d]) with Dsel the
       document rows the GPU argmax names for each (n, q) over ALL documents
       (zeros where it is -1), so the sum is checked over the whole batch.
    """
    Q = np.asarray(Q, dtype=np.float32)
    D_rows = np.asarray(D_rows, dtype=np.float32)
    Nq, Lq, d = Q.shape
    n = D_rows.shape[0]
    res = {}
    res["scores"] = _compare(scores_rows, O.maxsim_batched(Q, D_rows, lens_rows), "train scores")
    # eps-argmax
    am = np.asarray(am_rows)
    lens = np.asarray(lens_rows) if lens_rows is not None else np.full(n, D_rows.shape[1])
    bad = 0
    worst = 0.0
    for k in range(Nq):
        S = np.matmul(Q[k][None], D_rows.transpose(0, 2, 1))  # [n, Lq, Ld]
        pos = np.arange(D_rows.shape[1])
        S = np.where((pos[None, :] >= lens[:, None])[:, None, :], np.float32(-np.inf), S)
        rowmax = S.max(axis=2)
        a = am[k]
        empty = lens == 0
        bad += int(np.sum(a[empty] != -1))
        ne = ~empty
        a_ne = a[ne]
        in_range = (a_ne >= 0) & (a_ne < lens[ne][:, None])
        bad += int(np.sum(~in_range))
        picked = np.take_along_axis(S[ne], np.clip(a_ne, 0, S.shape[2] - 1)[:, :, None], axis=2)[:, :, 0]
        gap = rowmax[ne] - picked
        if gap.size:
            worst = max(worst, float(np.max(np.where(in_range, gap, 0.0))))
        bad += int(np.sum(in_range & (gap > eps)))
    res["argmax"] = {"checked": int(am.size), "max_abs_err": worst, "ok": bad == 0, "bad": bad}
    # dD of sampled documents for the GPU argmax
    g_rows = np.asarray(g_rows, dtype=np.float64)
    g_eff = np.where(np.isfinite(np.asarray(scores_rows)), g_rows, 0.0)
    _, wD = O.maxsim_grads(Q, D_rows, am, g_eff)
    res["dD"] = _compare(dD_rows, wD, "dD")
    # dQ rows over the whole batch
    g_all, Dsel = dq_want_inputs
    g_all = np.asarray(g_all, dtype=np.float64)
    want_q = []
    for r, (k, q) in enumerate(dq_rows_idx):
        want_q.append((g_all[k][:, None] * np.asarray(Dsel[r], dtype=np.float64)).sum(axis=0))
    res["dQ"] = _compare(dq_got, np.stack(want_q), "dQ")
    ok = all(v["ok"] for v in res.values())
    checked = sum(v["checked"] for v in res.values())
    err = max((v["max_abs_err"] or 0.0) for v in res.values())
    return {"checked": checked, "max_abs_err": err, "ok": ok, "parts": res}
