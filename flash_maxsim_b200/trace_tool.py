"""Per-event timeline of CTA 0 of one forward launch (trace builds only).

Builds libflashmaxsim_sm100_trace.so (the library with -DFM_TRACE: the lane-0
thread of each role of CTA 0 records (clock64, event code) pairs into a
device array, 4096 per channel), scores one batched shared-document call and
prints, per role, the median cycles between consecutive events.  The default
library has no trace code; this tool never touches it.

    python flash_maxsim_b200/trace_tool.py --docs 3000     # on a GPU box

Channels and event codes (csrc/fm_fwd.cuh):
  0, 5  MMA issuers (warps 1 and 11): 8/9 document chunks resident, 5/6 query
        stage wait, 1/2 accumulator slot wait, 3 MMAs issued, 4 slot
        committed, 7 query stage released
  1, 2  first warp of each epilogue set (warps 2 and 7): 1/2 slot wait,
        3 chunk maxima done, 5/6 pair barrier of the two sets
  3     query producer: 1/2 stage wait;  4  document producer: 1/2 slot wait, 3 issued
"""
from __future__ import annotations

import argparse
import collections
import ctypes
import os
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
TRACE_LIB = PKG_DIR / "libflashmaxsim_sm100_trace.so"
NAMES = {0: "issuer 0", 5: "issuer 1", 1: "epilogue set 0", 2: "epilogue set 1", 3: "query producer",
         4: "document producer"}


def build_trace_lib(force: bool = False) -> Path:
    sys.path.insert(0, str(PKG_DIR))
    import build as B  # the package's build script, loaded without importing the package

    if TRACE_LIB.exists() and not force and all(
            not p.exists() or p.stat().st_mtime <= TRACE_LIB.stat().st_mtime for p in B.DEPENDS):
        return TRACE_LIB
    cmd = [B.nvcc_path(), *B.NVCC_FLAGS, "-DFM_TRACE", *map(str, B.SOURCES), "-o", str(TRACE_LIB)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}")
    return TRACE_LIB


def segments(words):
    """Median cycles and counts between consecutive (code_a, code_b) events."""
    ev = [(int(w) >> 8, int(w) & 255) for w in words if int(w) != 0]
    seg = collections.defaultdict(list)
    for (ta, ca), (tb, cb) in zip(ev, ev[1:]):
        seg[(ca, cb)].append(tb - ta)
    return ev, seg


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--docs", type=int, default=3000)
    ap.add_argument("--nq", type=int, default=100)
    ap.add_argument("--lq", type=int, default=32)
    ap.add_argument("--ld", type=int, default=300)
    ap.add_argument("--dim", type=int, default=128)
    args = ap.parse_args()

    os.environ["FLASH_MAXSIM_LIB"] = str(build_trace_lib())
    sys.path.insert(0, str(REPO_DIR))
    import numpy as np
    import torch

    import flash_maxsim_b200 as fm

    lib = ctypes.CDLL(os.environ["FLASH_MAXSIM_LIB"])  # the same handle the package loaded
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    Q = torch.randn(args.nq, args.lq, args.dim, device=dev, generator=g).half()
    D = torch.randn(args.docs, args.ld, args.dim, device=dev, generator=g).half()
    for _ in range(3):
        fm.flash_maxsim_batched(Q, D)
    torch.cuda.synchronize()
    buf = (ctypes.c_ulonglong * (8 * 4096))()
    if lib.fm_trace_read(buf, 1) != 0:
        raise RuntimeError("fm_trace_read failed")
    fm.flash_maxsim_batched(Q, D)
    torch.cuda.synchronize()
    fm.check_status(dev)
    if lib.fm_trace_read(buf, 0) != 0:
        raise RuntimeError("fm_trace_read failed")
    words = np.frombuffer(buf, dtype=np.uint64).reshape(8, 4096)
    print(f"Q [{args.nq},{args.lq},{args.dim}] x D [{args.docs},{args.ld},{args.dim}] fp16, CTA 0")
    for ch, name in NAMES.items():
        ev, seg = segments(words[ch])
        if len(ev) < 2:
            continue
        starts = [t for t, c in ev if c == (5 if ch in (0, 5, 1, 2) else 1)]
        per = (ev[-1][0] - ev[0][0]) / max(1, len(starts))
        rows = ", ".join(f"{a}->{b}: {int(np.median(v))} (x{len(v)})"
                         for (a, b), v in sorted(seg.items()) if len(v) >= 8)
        print(f"ch {ch} {name}: {len(ev)} events, {per:.0f} cycles per query block (producers: per load); {rows}")


if __name__ == "__main__":
    main()
