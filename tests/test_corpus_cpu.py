"""Corpus files and per-rank shard loading on CPU: every rank of a world
gets exactly its contiguous document range, and the ranges tile the corpus."""
import json

import numpy as np
import torch


def _write(path, fmt, B=23, Ld=7, d=16):
    rng = np.random.default_rng(0)
    path.mkdir(parents=True, exist_ok=True)
    files = {"tokens": rng.integers(0, 255, (B, Ld, d)).astype(np.uint8)}
    if fmt == "int8":
        files["scales"] = rng.random((B, Ld)).astype(np.float16)
        files["mins"] = rng.random((B, Ld)).astype(np.float16)
    elif fmt == "fp8":
        files["scales"] = rng.random((B, Ld)).astype(np.float32)
    else:
        files["tokens"] = rng.standard_normal((B, Ld, d)).astype(np.float16)
    for k, v in files.items():
        np.save(path / f"{k}.npy", v)
    lens = rng.integers(0, Ld + 1, B).astype(np.int32)
    np.save(path / "lengths.npy", lens)
    (path / "meta.json").write_text(json.dumps({"format": fmt, "B": B, "Ld": Ld, "d": d}))
    return files, lens


def test_shards_tile_the_corpus(tmp_path):
    from flash_maxsim_b200.corpus import load_shard
    for fmt in ("fp16", "int8", "fp8"):
        files, lens = _write(tmp_path / fmt, fmt)
        for world in (1, 2, 3, 8):
            parts = [load_shard(tmp_path / fmt, r, world, device="cpu") for r in range(world)]
            assert parts[0]["lo"] == 0 and parts[-1]["hi"] == 23
            for a, b in zip(parts, parts[1:]):
                assert a["hi"] == b["lo"]
            for name, v in files.items():
                got = torch.cat([p[name] for p in parts]).numpy()
                np.testing.assert_array_equal(got, v)
            np.testing.assert_array_equal(torch.cat([p["lengths"] for p in parts]).numpy(), lens)
