"""The sampled full-size checker (oracle/sampled_check.py) on CPU: it passes
the oracle's own outputs and flags a perturbed score, a wrong argmax and a
wrong gradient row."""
import numpy as np

from oracle import maxsim_oracle as O
from oracle import sampled_check as SC


def test_sample_docs():
    idx = SC.sample_docs(1000, 10, seed=1)
    assert idx[0] == 0 and idx[-1] == 999 and len(set(idx)) == len(idx) and np.all(np.diff(idx) > 0)
    assert list(SC.sample_docs(3, 10)) == [0, 1, 2]


def test_check_scores_flags_errors():
    Q, D = O.seeded_inputs(0, (3, 8, 32), (12, 20, 32))
    lens = np.array([0, 5, 20] * 4, dtype=np.int32)
    want = O.maxsim_batched(Q, D, lens)
    assert SC.check_scores(Q, D, want, lens)["ok"]
    bad = want.copy()
    bad[1, 4] += 0.05
    assert not SC.check_scores(Q, D, bad, lens)["ok"]
    bad = want.copy()
    bad[0, 1] = -np.inf  # -inf only where the oracle has it
    assert not SC.check_scores(Q, D, bad, lens)["ok"]


def test_check_train_flags_errors():
    Nq, Lq, B, Ld, d = 2, 4, 6, 10, 16
    Q, D = O.seeded_inputs(1, (Nq, Lq, d), (B, Ld, d))
    lens = np.array([10, 0, 3, 7, 10, 1], dtype=np.int32)
    g = np.random.default_rng(2).standard_normal((Nq, B)).astype(np.float32)
    sc, am = [], []
    for n in range(Nq):
        s, a, _ = O.maxsim_argmax(Q[n], D, lens)
        sc.append(s)
        am.append(np.where((lens == 0)[:, None], -1, a))
    sc, am = np.stack(sc), np.stack(am)
    g_eff = np.where(np.isfinite(sc), g, 0.0)
    dQ, dD = O.maxsim_grads(Q, D, am, g_eff)
    rows = [(0, 0), (1, 3)]
    Dsel = []
    for n, q in rows:
        a = am[n, :, q]
        Dsel.append(np.where((a >= 0)[:, None], D[np.arange(B), np.clip(a, 0, None)].astype(np.float32), 0.0))
    args = dict(dq_rows_idx=rows, dq_want_inputs=(g_eff, Dsel))
    dq_got = np.stack([dQ[n, q] for n, q in rows])
    ok = SC.check_train(Q, D, lens, g, sc, am, dD, dq_got=dq_got, **args)
    assert ok["ok"], ok
    am_bad = am.copy()
    am_bad[0, 0, 0] = (am[0, 0, 0] + 1) % 10
    assert not SC.check_train(Q, D, lens, g, sc, am_bad, dD, dq_got=dq_got, **args)["parts"]["argmax"]["ok"]
    dD_bad = dD.copy()
    dD_bad[3, 0, 0] += 0.1
    assert not SC.check_train(Q, D, lens, g, sc, am, dD_bad, dq_got=dq_got, **args)["ok"]
    dq_bad = dq_got.copy()
    dq_bad[1, 5] += 0.1
    assert not SC.check_train(Q, D, lens, g, sc, am, dD, dq_got=dq_bad, **args)["ok"]
