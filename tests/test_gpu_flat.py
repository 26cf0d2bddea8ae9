"""Parity of the flat-token batched kernel (csrc/fm_flat.cuh), which is opt-in
(FLASH_MAXSIM_TUNE=flat=1, read once per process), so each case runs in a
child process with that setting and is checked against the oracle here."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import maxsim_oracle as O

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import json, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import flash_maxsim_b200 as fm
from oracle import maxsim_oracle as O
out = []
for Nq, Lq, B, Ld, d in json.loads(sys.argv[2]):
    Q, D = O.seeded_inputs(7 * Nq + Ld, (Nq, Lq, d), (B, Ld, d))
    got = fm.flash_maxsim_batched(torch.from_numpy(Q).cuda(), torch.from_numpy(D).cuda())
    fm.check_status()
    want = O.maxsim_batched(Q, D)
    err = np.abs(got.cpu().numpy() - want)
    ok = bool(np.all(err <= 1e-2 + 1e-3 * np.abs(want)))
    out.append([Nq, Lq, B, Ld, d, ok, float(err.max())])
print(json.dumps(out))
"""

CASES = [(4, 32, 300, 300, 128), (5, 64, 77, 150, 128), (4, 32, 97, 128, 128), (2, 96, 200, 257, 96),
         (3, 64, 50, 200, 64), (40, 128, 20, 300, 128), (16, 1024, 7, 1024, 128), (100, 32, 1000, 300, 128)]


@pytest.mark.gpu
def test_flat_kernel_vs_oracle():
    env = dict(os.environ, FLASH_MAXSIM_TUNE="flat=1", FLASH_MAXSIM_SYNC_CHECK="1")
    res = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), json.dumps(CASES)], env=env,
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    rows = json.loads(res.stdout.strip().splitlines()[-1])
    bad = [r for r in rows if not r[5]]
    assert not bad, f"flat kernel mismatches (Nq, Lq, B, Ld, d, ok, max_err): {bad}"
