"""Generate the golden vectors in tests/golden/ from the reference itself.

Imports the reference package (roipony/flash-maxsim 0.1.0) from a local
checkout and runs its own CPU-capable functions -- maxsim_naive,
maxsim_sparse_naive, quantize_int8, dequantize_int8 and torch autograd
through maxsim_naive -- on small seeded inputs. The outputs pin the numpy
oracle (oracle/maxsim_oracle.py) and the GPU kernels.

    python tests/golden/make_golden.py [--ref PATH_TO_REFERENCE_CHECKOUT]

Run once where the reference checkout exists; the .npz files are committed.
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from oracle.maxsim_oracle import seeded_inputs  # noqa: E402


def load_reference(ref_root: Path):
    pkg = ref_root / "flash_maxsim"
    spec = importlib.util.spec_from_file_location(
        "flash_maxsim_reference", pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["flash_maxsim_reference"] = mod
    spec.loader.exec_module(mod)
    return mod


def t(x):
    return torch.from_numpy(np.ascontiguousarray(x))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    ref = load_reference(Path(args.ref))
    print("reference version", ref.__version__)

    # 1. textual single query + variable lengths (incl. 0, 1 and Ld)
    Q, D = seeded_inputs(1, (32, 128), (24, 300, 128))
    lens = np.random.default_rng(2).integers(0, 301, 24).astype(np.int32)
    lens[:4] = [0, 1, 300, 299]
    s_full = ref.maxsim_naive(t(Q), t(D)).numpy()
    s_len = ref.maxsim_naive(t(Q), t(D), doc_lengths=t(lens)).numpy()
    np.savez_compressed(HERE / "textual.npz", Q=Q, D=D, lengths=lens, scores=s_full,
                        scores_len=s_len)

    # 2. batched = maxsim_naive per query (bench.py's own oracle loop)
    Qb, Db = seeded_inputs(3, (5, 32, 128), (20, 160, 128))
    sb = np.stack([ref.maxsim_naive(t(Qb[n]), t(Db)).numpy() for n in range(5)])
    np.savez_compressed(HERE / "batched.npz", Q=Qb, D=Db, scores=sb)

    # 3. INT8: quantize (bit-exact target) and scores on the dequantized docs
    Qi, Di = seeded_inputs(4, (32, 128), (16, 96, 128))
    u8, sc, mn = ref.quantize_int8(t(Di))
    deq = ref.dequantize_int8(u8, sc, mn)
    si = ref.maxsim_naive(t(Qi), deq).numpy()
    (Df32,) = seeded_inputs(5, (4, 33, 64), dtype=np.float32)  # fp32 input path
    u8f, scf, mnf = ref.quantize_int8(t(Df32))
    np.savez_compressed(HERE / "int8.npz", Q=Qi, D=Di, u8=u8.numpy(), scales=sc.numpy(),
                        mins=mn.numpy(), deq=deq.numpy(), scores=si, D32=Df32,
                        u8_32=u8f.numpy(), scales_32=scf.numpy(), mins_32=mnf.numpy())

    # 4. sparse: per-doc query subsets (the reference test's topk recipe)
    Qs, Ds = seeded_inputs(6, (32, 128), (24, 200, 128))
    g = torch.Generator().manual_seed(7)
    idx = torch.randn(24, 32, generator=g).topk(16, dim=1).indices.to(torch.int32)
    ss = ref.maxsim_sparse_naive(t(Qs), t(Ds), idx).numpy()
    np.savez_compressed(HERE / "sparse.npz", Q=Qs, D=Ds, indices=idx.numpy(), scores=ss)

    # 5. training: scores and gradients by autograd through maxsim_naive
    Qt, Dt = seeded_inputs(8, (16, 128), (10, 64, 128))
    qv = t(Qt).float().requires_grad_(True)
    dv = t(Dt).float().requires_grad_(True)
    st = ref.maxsim_naive(qv, dv)
    gs = torch.from_numpy(np.random.default_rng(9).standard_normal(10).astype(np.float32))
    (st * gs).sum().backward()
    np.savez_compressed(HERE / "train.npz", Q=Qt, D=Dt, grad_scores=gs.numpy(),
                        scores=st.detach().numpy(), dQ=qv.grad.numpy(), dD=dv.grad.numpy())

    # 6. large embedding dims (reference test_large_embedding_dim)
    out = {}
    for d in (256, 512, 1024, 2048):
        Ql, Dl = seeded_inputs(10 + d, (32, d), (4, 64, d))
        out[f"Q{d}"] = Ql
        out[f"D{d}"] = Dl
        out[f"s{d}"] = ref.maxsim_naive(t(Ql), t(Dl)).numpy()
    np.savez_compressed(HERE / "large_d.npz", **out)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
