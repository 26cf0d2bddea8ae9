"""Index-time corpus files and per-rank loading for document-sharded scoring.

A corpus directory holds the documents in one of the formats the scoring
kernels read, as plain .npy files (memory-mappable, no pickles):

    meta.json    {"format": "fp16" | "int8" | "fp8", "B", "Ld", "d"}
    tokens.npy   [B, Ld, d]  fp16 (fp16) or uint8 (int8 codes / e4m3 bit patterns)
    scales.npy   [B, Ld]     fp16 (int8) or fp32 (fp8)
    mins.npy     [B, Ld]     fp16 (int8 only)
    lengths.npy  [B]         int32 valid tokens per document

`build_corpus` writes one from batches of raw encoder output: each batch is
L2-normalised and quantised on the GPU in a single kernel pass
(fm_normalize_quantize_int8 / _fp8) and appended to the memory-mapped files.
`load_shard` gives rank r of N its contiguous document range
(sharded.shard_range) on its GPU: the files are memory-mapped, and the
range is streamed to the device through two pinned staging buffers on a
side stream, so reading the next piece from disk overlaps the copy of the
previous one. Nothing else of the corpus is read by that rank.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

FORMATS = ("fp16", "int8", "fp8")


def _files(fmt: str) -> tuple[str, ...]:
    return {"fp16": ("tokens",), "int8": ("tokens", "scales", "mins"), "fp8": ("tokens", "scales")}[fmt]


def _dtypes(fmt: str) -> dict:
    return {"fp16": {"tokens": np.float16},
            "int8": {"tokens": np.uint8, "scales": np.float16, "mins": np.float16},
            "fp8": {"tokens": np.uint8, "scales": np.float32}}[fmt]


def build_corpus(path, batches, fmt: str, B: int, Ld: int, d: int, device=None) -> Path:
    """Write a corpus of B documents from `batches`, an iterable of
    (embeddings [b, Ld, d] (any float dtype, CPU or CUDA), lengths [b]) in
    document order. fp16 documents are L2-normalised on the GPU; int8 and
    fp8 documents are normalised and quantised in one kernel pass."""
    from . import api
    if fmt not in FORMATS:
        raise ValueError(f"format {fmt!r} not in {FORMATS}")
    device = torch.device(device or "cuda")
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    dt = _dtypes(fmt)
    mm = {"tokens": np.lib.format.open_memmap(path / "tokens.npy", mode="w+", dtype=dt["tokens"], shape=(B, Ld, d))}
    for name in _files(fmt)[1:]:
        mm[name] = np.lib.format.open_memmap(path / f"{name}.npy", mode="w+", dtype=dt[name], shape=(B, Ld))
    lengths = np.zeros(B, dtype=np.int32)
    b0 = 0
    for emb, lens in batches:
        emb = emb.to(device)
        n = emb.shape[0]
        if b0 + n > B or tuple(emb.shape[1:]) != (Ld, d):
            raise ValueError(f"batch of shape {tuple(emb.shape)} does not fit a corpus of [{B}, {Ld}, {d}] at {b0}")
        if fmt == "fp16":
            out = {"tokens": F.normalize(emb.float(), dim=-1).half()}
        elif fmt == "int8":
            u8, sc, mn = api.quantize_int8(emb, normalize=True)
            out = {"tokens": u8, "scales": sc.squeeze(-1), "mins": mn.squeeze(-1)}
        else:
            codes, sc = api.quantize_fp8(emb, normalize=True)
            out = {"tokens": codes, "scales": sc.squeeze(-1)}
        for name, t in out.items():
            mm[name][b0:b0 + n] = t.cpu().numpy()
        lengths[b0:b0 + n] = torch.as_tensor(lens).cpu().numpy()
        b0 += n
    if b0 != B:
        raise ValueError(f"batches held {b0} documents, expected {B}")
    for m in mm.values():
        m.flush()
    np.save(path / "lengths.npy", lengths)
    (path / "meta.json").write_text(json.dumps({"format": fmt, "B": B, "Ld": Ld, "d": d}))
    return path


def corpus_meta(path) -> dict:
    return json.loads((Path(path) / "meta.json").read_text())


def _stream_rows(src: np.ndarray, dst: torch.Tensor, chunk_bytes: int) -> None:
    """Copy host rows src (a memory map) into the device tensor dst through
    two pinned staging buffers: while one piece is copied to the device on a
    side stream, the next is read from the map into the other buffer."""
    n = src.shape[0]
    if n == 0:
        return
    row_bytes = max(1, src[0].nbytes)
    rows = max(1, chunk_bytes // row_bytes)
    dev = dst.device
    with torch.cuda.device(dev):
        _stream_rows_on(src, dst, rows, dev)


def _stream_rows_on(src: np.ndarray, dst: torch.Tensor, rows: int, dev) -> None:
    n = src.shape[0]
    stream = torch.cuda.Stream(dev)
    stage = [torch.empty((rows,) + tuple(src.shape[1:]), dtype=dst.dtype, pin_memory=True) for _ in range(2)]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    busy = [False, False]
    for i, r0 in enumerate(range(0, n, rows)):
        k = i & 1
        m = min(rows, n - r0)
        if busy[k]:
            done[k].synchronize()  # the copy out of this buffer has finished
        stage[k][:m].numpy()[...] = src[r0:r0 + m]
        with torch.cuda.stream(stream):
            dst[r0:r0 + m].copy_(stage[k][:m], non_blocking=True)
            done[k].record(stream)
        busy[k] = True
    torch.cuda.current_stream(dev).wait_stream(stream)
    stream.synchronize()


def load_shard(path, rank: int = 0, world: int = 1, device=None, chunk_bytes: int = 256 << 20) -> dict:
    """This rank's documents [lo, hi) = shard_range(B, rank, world) of the
    corpus at `path`, on `device` (default: the current CUDA device).
    Returns {"format", "lo", "hi", "tokens", "lengths", + "scales", "mins"
    as the format has them}; tensors are shaped as the scoring API takes
    them (tokens [n, Ld, d], scales / mins [n, Ld], lengths int32 [n])."""
    from .sharded import shard_range
    meta = corpus_meta(path)
    fmt = meta["format"]
    lo, hi = shard_range(int(meta["B"]), rank, world)
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    tdt = {np.float16: torch.float16, np.uint8: torch.uint8, np.float32: torch.float32}
    out = {"format": fmt, "lo": lo, "hi": hi}
    for name in _files(fmt):
        src = np.load(Path(path) / f"{name}.npy", mmap_mode="r")[lo:hi]
        dst = torch.empty(src.shape, dtype=tdt[src.dtype.type], device=device)
        if device.type == "cuda":
            _stream_rows(src, dst, chunk_bytes)
        else:
            dst.numpy()[...] = src
        out[name] = dst
    out["lengths"] = torch.from_numpy(np.load(Path(path) / "lengths.npy")[lo:hi].copy()).to(device)
    return out


def score_shard(Q: torch.Tensor, shard: dict) -> torch.Tensor:
    """Score one query Q [Lq, d] (or a batch [Nq, Lq, d], fp16 format only)
    against a loaded shard with the kernel of its format."""
    from . import api
    fmt = shard["format"]
    if fmt == "fp16":
        if Q.dim() == 3:
            return api.flash_maxsim_batched(Q, shard["tokens"], shard["lengths"])
        return api.flash_maxsim(Q, shard["tokens"], shard["lengths"])
    if fmt == "int8":
        return api.flash_maxsim_int8(Q, shard["tokens"], shard["scales"], shard["mins"], shard["lengths"])
    return api.flash_maxsim_fp8(Q, shard["tokens"], shard["scales"], shard["lengths"])
