"""Public MaxSim API, call-compatible with flash_maxsim 0.1.0 (flash_maxsim/__init__.py:3-5).

Every scoring function runs the hand-written sm_100a kernels of
libflashmaxsim_sm100.so; inputs must be CUDA tensors (there is no CPU path).
`maxsim_naive`, `maxsim_sparse_naive` and `dequantize_int8` are the
reference's plain-torch helpers and stay plain torch, as in the reference.

Error behaviour follows the reference: shape mismatches raise AssertionError
(flash_maxsim/flash_maxsim.py:223,236,239,242; flash_maxsim_quant.py:22,113;
flash_maxsim_sparse.py:115,119); a host-side launch error raises
RuntimeError / ValueError; device-side errors land in the status word read by
`check_status()`, and (without a synchronisation) at the next call on the
same device once an asynchronous copy of the status word has reached the host.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib
from ._lib import lib


# ---------------------------------------------------------------------------
# input preparation
# ---------------------------------------------------------------------------

def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(
                "flash_maxsim_b200 scores CUDA tensors only (the kernels are sm_100a CUDA); "
                f"got a tensor on {t.device}"
            )


def _pad_last(t: torch.Tensor, mult: int) -> torch.Tensor:
    d = t.shape[-1]
    pad = (-d) % mult
    return F.pad(t, (0, pad)) if pad else t


def _aligned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _half(t: torch.Tensor, mult: int = 8) -> torch.Tensor:
    """Reference casting (`.contiguous().half()`), plus zero padding of the
    embedding dimension to a multiple of `mult` (zeros add nothing to a dot
    product) and 16-byte alignment for TMA."""
    return _aligned(_pad_last(t.half(), mult))


def _lengths(doc_lengths, n: int, Ld: int, device) -> torch.Tensor | None:
    # _default_lengths (flash_maxsim/flash_maxsim.py:211-214); None means "all Ld"
    if doc_lengths is None:
        return None
    if not torch.is_tensor(doc_lengths):
        doc_lengths = torch.as_tensor(doc_lengths)
    lens = doc_lengths.to(device=device, dtype=torch.int32).contiguous()
    assert lens.numel() == n, f"doc_lengths has {lens.numel()} entries, expected {n}"
    return lens


def _after_call(device):
    _lib.after_call(device)


def _before_call(device):
    # an error recorded by an earlier call on this device surfaces here
    _lib.poll_status(device)


def _fwd(Q3: torch.Tensor, D2: torch.Tensor, lengths, Nq, B, Lq, Ld, shared: bool,
         save_argmax: bool):
    """Launch fm_maxsim_fwd. Q3: [Nq, Lq, d'] fp16, D2: [docs, Ld, d'] fp16."""
    dev = Q3.device
    scores = torch.empty(Nq, B, device=dev, dtype=torch.float32)
    argmax = (torch.empty(Nq * B, Lq, device=dev, dtype=torch.int32) if save_argmax else None)
    if B == 0:
        return scores, argmax
    d = Q3.shape[-1]
    _before_call(dev)
    with _lib.on_device(dev):
        rc = lib.fm_maxsim_fwd(
            Q3.data_ptr(), D2.data_ptr(), _lib.ptr(lengths), scores.data_ptr(),
            _lib.ptr(argmax), Nq, B, Lq, Ld, d, 1 if shared else 0,
            _lib.status_word(dev).data_ptr(), _lib.stream_of(dev))
    _lib.check(rc, "fm_maxsim_fwd")
    _after_call(dev)
    return scores, argmax


def _degenerate(Nq, B, Lq, Ld, device):
    """Scores when the kernel has nothing to do: no query tokens sum to 0,
    no document tokens give max = -inf (as the reference's loops do)."""
    if Lq == 0:
        return torch.zeros(Nq, B, device=device, dtype=torch.float32)
    return torch.full((Nq, B), float("-inf"), device=device, dtype=torch.float32)


# ---------------------------------------------------------------------------
# fp16 forward (flash_maxsim/flash_maxsim.py:221-250)
# ---------------------------------------------------------------------------

def flash_maxsim(Q: torch.Tensor, D: torch.Tensor, doc_lengths=None) -> torch.Tensor:
    """Compute MaxSim scores. Q: [Lq, d], D: [B, Ld, d] -> [B] fp32.

    score[b] = sum_q max_{t < doc_lengths[b]} <Q[q], D[b, t]>; inputs are cast
    to fp16 like the reference (flash_maxsim/flash_maxsim.py:221-230).
    """
    assert Q.dim() == 2 and D.dim() == 3 and Q.shape[1] == D.shape[2]
    _require_cuda(Q, D)
    Lq, d = Q.shape
    B, Ld, _ = D.shape
    lengths = _lengths(doc_lengths, B, Ld, D.device)
    if Lq == 0 or Ld == 0:
        return _degenerate(1, B, Lq, Ld, D.device).squeeze(0)
    Q3 = _half(Q.unsqueeze(0))
    D2 = _half(D)
    scores, _ = _fwd(Q3, D2, lengths, 1, B, Lq, Ld, True, False)
    return scores.squeeze(0)


def flash_maxsim_batched(Q: torch.Tensor, D: torch.Tensor, doc_lengths=None,
                         shared_docs: bool = True) -> torch.Tensor:
    """Batched MaxSim. Q: [Nq, Lq, d], D: [B, Ld, d] -> [Nq, B] fp32.

    shared_docs=False takes per-query documents D: [Nq, B, Ld, d] and
    doc_lengths of Nq*B entries (flash_maxsim/flash_maxsim.py:233-250).
    Every document is read from HBM once for the whole query batch.
    """
    assert Q.dim() == 3 and Q.shape[2] == D.shape[-1]
    _require_cuda(Q, D)
    Nq, Lq, d = Q.shape
    if shared_docs:
        assert D.dim() == 3
        B, Ld, _ = D.shape
    else:
        assert D.dim() == 4 and D.shape[0] == Nq
        _, B, Ld, _ = D.shape
        D = D.reshape(Nq * B, Ld, d)
    total = B if shared_docs else Nq * B
    lengths = _lengths(doc_lengths, total, Ld, D.device)
    if Nq == 0:
        return torch.empty(0, B, device=D.device, dtype=torch.float32)
    if Lq == 0 or Ld == 0:
        return _degenerate(Nq, B, Lq, Ld, D.device)
    scores, _ = _fwd(_half(Q), _half(D), lengths, Nq, B, Lq, Ld, shared_docs, False)
    return scores


_copy_streams: dict = {}


def _copy_stream(device) -> torch.cuda.Stream:
    """One host-to-device copy stream per device, created on first use."""
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    if idx not in _copy_streams:
        _copy_streams[idx] = torch.cuda.Stream(device=idx)
    return _copy_streams[idx]


def host_pieces(B: int, doc_bytes: int, piece_bytes: int) -> tuple[int, int]:
    """Documents per piece and number of pieces for streaming B documents of
    doc_bytes each in pieces of at most piece_bytes (at least one document
    per piece; piece i covers documents [i * piece, min(B, (i + 1) * piece)))."""
    piece = max(1, min(B, piece_bytes // max(1, doc_bytes)))
    return piece, (B + piece - 1) // piece


def flash_maxsim_batched_from_host(Q: torch.Tensor, D_host: torch.Tensor, doc_lengths=None,
                                   piece_bytes: int = 512 << 20, nbuf: int = 3,
                                   device=None) -> torch.Tensor:
    """flash_maxsim_batched over shared documents that stay in host memory:
    Q [Nq, Lq, d] (host or device), D_host [B, Ld, d] on the CPU -> [Nq, B]
    fp32 on the GPU (`device`, else Q's device if it is a CUDA tensor, else
    the current device).

    The documents cross PCIe in pieces of about `piece_bytes` on a copy
    stream, through `nbuf` device buffers, while the pieces already copied
    are scored on the current stream: the copies hide the scoring, and the
    GPU holds nbuf pieces instead of the whole corpus (a corpus larger than
    device memory can be scored). Each document is scored on its own, so the
    scores equal flash_maxsim_batched's on the whole corpus. D_host should be
    pinned (`pin_memory()`); from pageable memory every copy waits for the
    host and nothing overlaps. The call returns once everything is enqueued.
    """
    if device is None:
        device = Q.device if Q.is_cuda else torch.device("cuda", torch.cuda.current_device())
    dev = torch.device(device)
    if D_host.is_cuda:
        return flash_maxsim_batched(Q.to(dev), D_host, doc_lengths)
    assert Q.dim() == 3 and D_host.dim() == 3 and Q.shape[2] == D_host.shape[2]
    assert nbuf >= 1 and piece_bytes >= 1
    Nq, Lq, d = Q.shape
    B, Ld, _ = D_host.shape
    q = Q.to(dev, non_blocking=True)
    lengths = None
    if doc_lengths is not None:
        lengths = torch.as_tensor(doc_lengths).to(dev, non_blocking=True)
        assert lengths.numel() == B, "doc_lengths needs one entry per document"
    piece, npieces = host_pieces(B, Ld * d * D_host.element_size(), piece_bytes)
    if Nq == 0 or npieces <= 1:
        D = D_host.to(dev, non_blocking=True)
        return flash_maxsim_batched(q, D, lengths)
    out = torch.empty(Nq, B, dtype=torch.float32, device=dev)
    main = torch.cuda.current_stream(dev)
    cs = _copy_stream(dev)
    cs.wait_stream(main)  # the buffers below may reuse memory that queued work still reads
    bufs = [torch.empty((piece, Ld, d), dtype=D_host.dtype, device=dev)
            for _ in range(min(nbuf, npieces))]
    freed = [None] * len(bufs)  # event after the last scoring that read each buffer
    for i in range(npieces):
        b0, b1 = i * piece, min(B, (i + 1) * piece)
        k = i % len(bufs)
        buf = bufs[k][:b1 - b0]
        with torch.cuda.stream(cs):
            if freed[k] is not None:
                cs.wait_event(freed[k])
            buf.copy_(D_host[b0:b1], non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(cs)
        main.wait_event(ready)
        out[:, b0:b1] = flash_maxsim_batched(q, buf, None if lengths is None else lengths[b0:b1])
        ev = torch.cuda.Event()
        ev.record(main)
        freed[k] = ev
    return out


# ---------------------------------------------------------------------------
# packed (unpadded) documents
# ---------------------------------------------------------------------------

def flash_maxsim_packed(Q: torch.Tensor, D_tokens: torch.Tensor, cu_seqlens, max_len: int | None = None):
    """MaxSim over packed documents: document b is rows
    cu_seqlens[b]:cu_seqlens[b+1] of D_tokens [T, d] (ragged encoder output
    concatenated, no padding). Q: [Lq, d] -> [B] or [Nq, Lq, d] -> [Nq, B] fp32.

    Equal to flash_maxsim(_batched) on the same documents padded to
    [B, max_len, d] with doc_lengths = diff(cu_seqlens). `max_len` must bound
    every length (None: computed here, which synchronises with the device)."""
    assert Q.dim() in (2, 3) and D_tokens.dim() == 2 and Q.shape[-1] == D_tokens.shape[1]
    _require_cuda(Q, D_tokens)
    single = Q.dim() == 2
    Q3 = Q.unsqueeze(0) if single else Q
    Nq, Lq, d = Q3.shape
    cu = cu_seqlens if torch.is_tensor(cu_seqlens) else torch.as_tensor(cu_seqlens)
    cu = cu.to(device=D_tokens.device, dtype=torch.int32).contiguous()
    assert cu.dim() == 1 and cu.numel() >= 1
    B = cu.numel() - 1
    T = D_tokens.shape[0]
    dev = D_tokens.device
    if max_len is None:
        max_len = int((cu[1:] - cu[:-1]).max().item()) if B > 0 else 1
    max_len = max(int(max_len), 1)
    if B == 0 or Nq == 0:
        out = torch.empty(Nq, B, device=dev, dtype=torch.float32)
        return out.squeeze(0) if single else out
    if Lq == 0 or T == 0:
        out = _degenerate(Nq, B, Lq, 0 if T == 0 else max_len, dev)
        return out.squeeze(0) if single else out
    Qh, Dh = _half(Q3), _half(D_tokens)
    scores = torch.empty(Nq, B, device=dev, dtype=torch.float32)
    _before_call(dev)
    with _lib.on_device(dev):
        rc = lib.fm_maxsim_packed_fwd(Qh.data_ptr(), Dh.data_ptr(), cu.data_ptr(), scores.data_ptr(), None,
                                      Nq, B, Lq, max_len, Qh.shape[-1], T, _lib.status_word(dev).data_ptr(),
                                      _lib.stream_of(dev))
    _lib.check(rc, "fm_maxsim_packed_fwd")
    _after_call(dev)
    return scores.squeeze(0) if single else scores


def pack_documents(D: torch.Tensor, doc_lengths):
    """Padded [B, Ld, d] documents + lengths -> (D_tokens [sum(len), d],
    cu_seqlens int32 [B + 1]): the packed layout flash_maxsim_packed reads."""
    assert D.dim() == 3
    B, Ld, d = D.shape
    lens = torch.as_tensor(doc_lengths, device=D.device).to(torch.int64).clamp(0, Ld)
    cu = torch.zeros(B + 1, dtype=torch.int64, device=D.device)
    cu[1:] = torch.cumsum(lens, 0)
    mask = torch.arange(Ld, device=D.device)[None, :] < lens[:, None]
    return D[mask].contiguous(), cu.to(torch.int32)


# ---------------------------------------------------------------------------
# top-k (callers of the reference: examples/demo.py:126-134, benchmarks/bench.py:36)
# ---------------------------------------------------------------------------

def _topk_workspace(Nq: int, k: int, device) -> torch.Tensor:
    nbytes = int(lib.fm_topk_workspace_size(Nq, k))
    if nbytes <= 0:
        raise ValueError(f"top-k workspace unavailable for Nq={Nq}, k={k} (1 <= k <= 1024)")
    return torch.empty(-(-nbytes // 16) * 4, dtype=torch.float32, device=device)


def flash_maxsim_batched_topk(Q: torch.Tensor, D: torch.Tensor, k: int, doc_lengths=None):
    """The k best shared documents of every query: Q [Nq, Lq, d], D [B, Ld, d]
    -> (values fp32 [Nq, k], document ids int64 [Nq, k]).

    Same scores as flash_maxsim_batched; the scoring kernel keeps each query's
    k best documents per CTA and one merge kernel combines them, so the
    [Nq, B] matrix is never sorted. Order: score descending, ties by the lower
    document id. 1 <= k <= min(B, 1024)."""
    assert Q.dim() == 3 and D.dim() == 3 and Q.shape[2] == D.shape[2]
    _require_cuda(Q, D)
    Nq, Lq, d = Q.shape
    B, Ld, _ = D.shape
    k = int(k)
    assert 1 <= k <= B, f"k={k} outside [1, {B}]"
    lengths = _lengths(doc_lengths, B, Ld, D.device)
    dev = D.device
    if Nq == 0:
        return (torch.empty(0, k, device=dev, dtype=torch.float32),
                torch.empty(0, k, device=dev, dtype=torch.int64))
    if Lq == 0 or Ld == 0:
        return topk_scores(_degenerate(Nq, B, Lq, Ld, dev), k)
    Qh, Dh = _half(Q), _half(D)
    scores = torch.empty(Nq, B, device=dev, dtype=torch.float32)
    vals = torch.empty(Nq, k, device=dev, dtype=torch.float32)
    idx = torch.empty(Nq, k, device=dev, dtype=torch.int64)
    ws = _topk_workspace(Nq, k, dev)
    _before_call(dev)
    with _lib.on_device(dev):
        rc = lib.fm_maxsim_topk(Qh.data_ptr(), Dh.data_ptr(), _lib.ptr(lengths), scores.data_ptr(), k,
                                vals.data_ptr(), idx.data_ptr(), Nq, B, Lq, Ld, Qh.shape[-1],
                                ws.data_ptr(), ws.numel() * 4, _lib.status_word(dev).data_ptr(),
                                _lib.stream_of(dev))
    _lib.check(rc, "fm_maxsim_topk")
    _after_call(dev)
    return vals, idx


def flash_maxsim_topk(Q: torch.Tensor, D: torch.Tensor, k: int, doc_lengths=None):
    """The k best documents for one query: Q [Lq, d], D [B, Ld, d] ->
    (values fp32 [k], document ids int64 [k]); see flash_maxsim_batched_topk."""
    assert Q.dim() == 2
    v, i = flash_maxsim_batched_topk(Q.unsqueeze(0), D, k, doc_lengths)
    return v.squeeze(0), i.squeeze(0)


def topk_scores(scores: torch.Tensor, k: int, id_offset: int = 0):
    """GPU top-k of any score matrix [Nq, B] (or vector [B]), e.g. from
    flash_maxsim_int8 or flash_maxsim_sparse: (values, ids + id_offset),
    score descending, ties by the lower id."""
    _require_cuda(scores)
    vec = scores.dim() == 1
    s2 = scores.unsqueeze(0) if vec else scores
    assert s2.dim() == 2
    Nq, B = s2.shape
    k = int(k)
    assert 1 <= k <= B, f"k={k} outside [1, {B}]"
    s2 = s2.float().contiguous()
    dev = s2.device
    vals = torch.empty(Nq, k, device=dev, dtype=torch.float32)
    idx = torch.empty(Nq, k, device=dev, dtype=torch.int64)
    if Nq:
        ws = _topk_workspace(Nq, k, dev)
        with _lib.on_device(dev):
            rc = lib.fm_topk_select(s2.data_ptr(), Nq, B, k, int(id_offset), vals.data_ptr(), idx.data_ptr(),
                                    ws.data_ptr(), ws.numel() * 4, _lib.stream_of(dev))
        _lib.check(rc, "fm_topk_select")
    return (vals.squeeze(0), idx.squeeze(0)) if vec else (vals, idx)


def topk_merge_candidates(values: torch.Tensor, ids: torch.Tensor, k: int):
    """Merge per-part candidate lists values/ids [Nq, parts, k'] (ids < 0 =
    none; ids below 2**31) into the k best per query, on the GPU."""
    _require_cuda(values, ids)
    assert values.dim() == 3 and values.shape == ids.shape
    Nq, parts, kk = values.shape
    k = int(k)
    assert 1 <= k <= 1024
    v = values.float()
    i = ids.to(torch.int32)
    if kk < k:  # pad each part's list to k entries
        v = F.pad(v, (0, k - kk), value=float("-inf"))
        i = F.pad(i, (0, k - kk), value=-1)
    elif kk > k:
        v, i = v[..., :k], i[..., :k]  # lists are sorted: the first k suffice
    v, i = v.contiguous(), i.contiguous()
    dev = v.device
    vals = torch.empty(Nq, k, device=dev, dtype=torch.float32)
    idx = torch.empty(Nq, k, device=dev, dtype=torch.int64)
    if Nq:
        with _lib.on_device(dev):
            rc = lib.fm_topk_merge(v.data_ptr(), i.data_ptr(), Nq, parts, k, vals.data_ptr(), idx.data_ptr(),
                                   _lib.stream_of(dev))
        _lib.check(rc, "fm_topk_merge")
    return vals, idx


# ---------------------------------------------------------------------------
# training (flash_maxsim/flash_maxsim.py:253-291)
# ---------------------------------------------------------------------------

class _FlashMaxSimFn(torch.autograd.Function):
    """Forward saves the per-row argmax; backward scatters/gathers through it
    (the reference's _FlashMaxSimFn, flash_maxsim/flash_maxsim.py:253-286),
    extended to query batches and variable-length documents."""

    @staticmethod
    def forward(ctx, Q, D, doc_lengths):
        single = Q.dim() == 2
        Q3 = Q.unsqueeze(0) if single else Q
        Nq, Lq, d = Q3.shape
        B, Ld, _ = D.shape
        Qh = _half(Q3)
        Dh = _half(D)
        lengths = _lengths(doc_lengths, B, Ld, D.device)
        scores, argmax = _fwd(Qh, Dh, lengths, Nq, B, Lq, Ld, True, True)
        ctx.save_for_backward(Qh, Dh, argmax)
        ctx.meta = (single, Nq, B, Lq, Ld, d, Q.dtype, D.dtype)
        return scores.squeeze(0) if single else scores

    @staticmethod
    def backward(ctx, grad_scores):
        Qh, Dh, argmax = ctx.saved_tensors
        single, Nq, B, Lq, Ld, d, q_dtype, d_dtype = ctx.meta
        g = grad_scores.reshape(Nq, B).contiguous().float()
        dp = Qh.shape[-1]
        grad_Q = torch.empty(Nq, Lq, dp, device=Qh.device, dtype=torch.float16)
        grad_D = torch.empty(B, Ld, dp, device=Dh.device, dtype=torch.float16)
        dev = Qh.device
        ws_bytes = int(lib.fm_maxsim_bwd_workspace_size(Nq, B, Lq, Ld, dp))
        ws = torch.empty(max(ws_bytes, 0) // 4, device=dev, dtype=torch.float32) if ws_bytes > 0 else None
        _before_call(dev)
        with _lib.on_device(dev):
            rc = lib.fm_maxsim_bwd(
                Qh.data_ptr(), Dh.data_ptr(), argmax.data_ptr(), g.data_ptr(),
                grad_Q.data_ptr(), grad_D.data_ptr(), Nq, B, Lq, Ld, dp,
                _lib.ptr(ws), ws_bytes, _lib.stream_of(dev))
        _lib.check(rc, "fm_maxsim_bwd")
        _after_call(dev)
        grad_Q = grad_Q[..., :d]
        grad_D = grad_D[..., :d]
        if single:
            grad_Q = grad_Q.squeeze(0)
        gq = grad_Q.to(q_dtype) if ctx.needs_input_grad[0] else None
        gd = grad_D.to(d_dtype) if ctx.needs_input_grad[1] else None
        return gq, gd, None


def flash_maxsim_train(Q: torch.Tensor, D: torch.Tensor, doc_lengths=None) -> torch.Tensor:
    """MaxSim with autograd backward. Q: [Lq, d] -> [B] (reference signature),
    or Q: [Nq, Lq, d] -> [Nq, B]; D: [B, Ld, d]; optional doc_lengths [B].

    Gradients: dQ[q] = sum_b g_b D[b, argmax], dD[b, argmax] += g_b Q[q],
    accumulated in fp32 in a fixed order and returned in the input dtype.
    """
    assert Q.dim() in (2, 3) and D.dim() == 3 and Q.shape[-1] == D.shape[2]
    _require_cuda(Q, D)
    assert Q.shape[-2] >= 1 and D.shape[1] >= 1
    return _FlashMaxSimFn.apply(Q, D, doc_lengths)


def maxsim_naive(Q: torch.Tensor, D: torch.Tensor, doc_lengths=None) -> torch.Tensor:
    """Reference PyTorch MaxSim (flash_maxsim/flash_maxsim.py:294-301).
    Q: [Lq, d], D: [B, Ld, d] -> [B]; fp32 einsum, -inf past doc_lengths."""
    sim = torch.einsum("qd,bld->bql", Q.float(), D.float())
    if doc_lengths is not None:
        pos = torch.arange(D.shape[1], device=D.device)
        mask = pos[None, None, :] >= doc_lengths.to(D.device)[:, None, None]
        sim = sim.masked_fill(mask, float("-inf"))
    return sim.max(dim=2).values.sum(dim=1)


# ---------------------------------------------------------------------------
# INT8 (flash_maxsim/flash_maxsim_quant.py)
# ---------------------------------------------------------------------------

_QDTYPE = {torch.float16: _lib.FM_DTYPE_F16, torch.float32: _lib.FM_DTYPE_F32,
           torch.bfloat16: _lib.FM_DTYPE_BF16}


def quantize_int8(D: torch.Tensor, normalize: bool = False):
    """Per-token affine INT8 quantisation (flash_maxsim/flash_maxsim_quant.py:11-28).

    D: [B, Ld, d] -> (uint8 [B, Ld, d], scales fp16 [B, Ld, 1], mins fp16 [B, Ld, 1]),
    bit-identical to the reference formula, computed by one CUDA kernel pass.
    normalize=True (index time): every token row is first L2-normalised in the
    same pass (see normalize_quantize_int8).
    """
    assert D.dim() == 3
    _require_cuda(D)
    fn = lib.fm_normalize_quantize_int8 if normalize else lib.fm_quantize_int8
    B, Ld, d = D.shape
    x = D if D.dtype in _QDTYPE else D.float()
    # the kernel reads 8 elements per lane: pad rows with their own first
    # element (changes neither min nor max), then drop the padded columns
    pad = (-d) % 8
    if pad and normalize:
        raise ValueError(f"normalize=True needs d % 8 == 0 (got d={d})")
    if pad:
        x = torch.cat([x, x[..., :1].expand(B, Ld, pad)], dim=-1)
    x = _aligned(x)
    dp = d + pad
    u8 = torch.empty(B, Ld, dp, device=D.device, dtype=torch.uint8)
    scales = torch.empty(B, Ld, 1, device=D.device, dtype=torch.float16)
    mins = torch.empty(B, Ld, 1, device=D.device, dtype=torch.float16)
    rows = B * Ld
    if rows:
        _before_call(D.device)
        with _lib.on_device(D.device):
            rc = fn(x.data_ptr(), _QDTYPE[x.dtype], u8.data_ptr(), scales.data_ptr(), mins.data_ptr(), rows, dp,
                    _lib.stream_of(D.device))
        _lib.check(rc, "fm_normalize_quantize_int8" if normalize else "fm_quantize_int8")
        _after_call(D.device)
    if pad:
        u8 = u8[..., :d].contiguous()
    return u8, scales, mins


def dequantize_int8(D_uint8: torch.Tensor, scales: torch.Tensor, mins: torch.Tensor) -> torch.Tensor:
    """Reconstruct fp32 values u * scale + min (flash_maxsim/flash_maxsim_quant.py:31-33)."""
    return D_uint8.float() * scales.float() + mins.float()


def flash_maxsim_int8(Q: torch.Tensor, D_uint8: torch.Tensor, scales: torch.Tensor,
                      mins: torch.Tensor, doc_lengths=None) -> torch.Tensor:
    """Fused dequant + MaxSim. Q: [Lq, d], D_uint8: [B, Ld, d] -> [B] fp32
    (flash_maxsim/flash_maxsim_quant.py:105-142). scales/mins: [B, Ld, 1] or [B, Ld].

    The tensor cores multiply Q by the exact integers u; the per-token map
    scale * <q, u> + min * sum(q) is applied in fp32 in the epilogue.
    """
    assert Q.dim() == 2 and D_uint8.dim() == 3 and Q.shape[1] == D_uint8.shape[2]
    _require_cuda(Q, D_uint8, scales, mins)
    Lq, d = Q.shape
    B, Ld, _ = D_uint8.shape
    if scales.dim() == 3:
        scales = scales.squeeze(-1)
    if mins.dim() == 3:
        mins = mins.squeeze(-1)
    lengths = _lengths(doc_lengths, B, Ld, D_uint8.device)
    if Lq == 0 or Ld == 0:
        return _degenerate(1, B, Lq, Ld, D_uint8.device).squeeze(0)
    # zero-padding both Q and the codes keeps every dot product unchanged
    Qh = _half(Q, 16)
    Du = _aligned(_pad_last(D_uint8.to(torch.uint8), 16))
    sc = _aligned(scales.half())
    mn = _aligned(mins.half())
    assert sc.shape == (B, Ld) and mn.shape == (B, Ld)
    scores = torch.empty(B, device=Q.device, dtype=torch.float32)
    if B == 0:
        return scores
    dev = Q.device
    _before_call(dev)
    with _lib.on_device(dev):
        rc = lib.fm_maxsim_int8_fwd(Qh.data_ptr(), Du.data_ptr(), sc.data_ptr(), mn.data_ptr(),
                                    _lib.ptr(lengths), scores.data_ptr(), B, Lq, Ld,
                                    Qh.shape[-1], _lib.status_word(dev).data_ptr(),
                                    _lib.stream_of(dev))
    _lib.check(rc, "fm_maxsim_int8_fwd")
    _after_call(dev)
    return scores


# ---------------------------------------------------------------------------
# FP8 (e4m3) document storage: the INT8 path's sibling with one scale per token
# ---------------------------------------------------------------------------

def quantize_fp8(D: torch.Tensor, normalize: bool = False):
    """Per-token e4m3 quantisation on the GPU: D [B, Ld, d] (fp16 / bf16 /
    fp32) -> (codes uint8 [B, Ld, d] holding e4m3 bit patterns, scales fp32
    [B, Ld, 1]) with scale = max|x| / 448 (1 for an all-zero token) and
    code = e4m3(x / scale), round-to-nearest-even. normalize=True (index
    time): every token row is first L2-normalised in the same pass."""
    assert D.dim() == 3
    _require_cuda(D)
    fn = lib.fm_normalize_quantize_fp8 if normalize else lib.fm_quantize_fp8
    B, Ld, d = D.shape
    x = D if D.dtype in _QDTYPE else D.float()
    pad = (-d) % 8
    if pad:
        x = F.pad(x, (0, pad))  # zeros change no row's max |x| and no norm
    x = _aligned(x)
    dp = d + pad
    codes = torch.empty(B, Ld, dp, device=D.device, dtype=torch.uint8)
    scales = torch.empty(B, Ld, 1, device=D.device, dtype=torch.float32)
    rows = B * Ld
    if rows:
        _before_call(D.device)
        with _lib.on_device(D.device):
            rc = fn(x.data_ptr(), _QDTYPE[x.dtype], codes.data_ptr(), scales.data_ptr(), rows, dp,
                    _lib.stream_of(D.device))
        _lib.check(rc, "fm_normalize_quantize_fp8" if normalize else "fm_quantize_fp8")
        _after_call(D.device)
    if pad:
        codes = codes[..., :d].contiguous()
    return codes, scales


def dequantize_fp8(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Reconstruct fp32 values e4m3(code) * scale (plain torch)."""
    return codes.view(torch.float8_e4m3fn).float() * scales.float()


def flash_maxsim_fp8(Q: torch.Tensor, D_fp8: torch.Tensor, scales: torch.Tensor, doc_lengths=None) -> torch.Tensor:
    """MaxSim on e4m3 documents. Q: [Lq, d] (Lq <= 64), D_fp8: uint8 [B, Ld, d]
    e4m3 codes, scales: [B, Ld, 1] or [B, Ld] -> [B] fp32, equal to
    maxsim_naive(Q, dequantize_fp8(D_fp8, scales)) within fp32 rounding."""
    assert Q.dim() == 2 and D_fp8.dim() == 3 and Q.shape[1] == D_fp8.shape[2]
    _require_cuda(Q, D_fp8, scales)
    Lq, d = Q.shape
    B, Ld, _ = D_fp8.shape
    assert Lq <= 64, "the FP8 path scores queries of at most 64 tokens"
    if scales.dim() == 3:
        scales = scales.squeeze(-1)
    lengths = _lengths(doc_lengths, B, Ld, D_fp8.device)
    if Lq == 0 or Ld == 0:
        return _degenerate(1, B, Lq, Ld, D_fp8.device).squeeze(0)
    Qh = _half(Q, 16)
    Du = _aligned(_pad_last(D_fp8.view(torch.uint8) if D_fp8.dtype != torch.uint8 else D_fp8, 16))
    sc = _aligned(scales.float())
    assert sc.shape == (B, Ld)
    assert Qh.shape[-1] <= 256, "the FP8 path supports d <= 256"
    scores = torch.empty(B, device=Q.device, dtype=torch.float32)
    if B == 0:
        return scores
    dev = Q.device
    _before_call(dev)
    with _lib.on_device(dev):
        rc = lib.fm_maxsim_fp8_fwd(Qh.data_ptr(), Du.data_ptr(), sc.data_ptr(), _lib.ptr(lengths), scores.data_ptr(),
                                   B, Lq, Ld, Qh.shape[-1], _lib.status_word(dev).data_ptr(), _lib.stream_of(dev))
    _lib.check(rc, "fm_maxsim_fp8_fwd")
    _after_call(dev)
    return scores


# ---------------------------------------------------------------------------
# sparse (flash_maxsim/flash_maxsim_sparse.py)
# ---------------------------------------------------------------------------

def flash_maxsim_sparse(Q: torch.Tensor, D: torch.Tensor, indices: torch.Tensor,
                        doc_lengths=None) -> torch.Tensor:
    """Sparse MaxSim with per-doc query-token selection
    (flash_maxsim/flash_maxsim_sparse.py:98-140).

    Q: [Lq, d] shared query, D: [B, Ld, d], indices: [B, K] query-token ids per
    doc, doc_lengths: optional [B]. Returns [B] fp32:
    score[b] = sum_k max_{t < len_b} <Q[indices[b, k]], D[b, t]>.
    """
    assert Q.dim() == 2 and D.dim() == 3 and indices.dim() == 2
    _require_cuda(Q, D, indices)
    Lq, d = Q.shape
    B, Ld, _ = D.shape
    _, K = indices.shape
    assert indices.shape[0] == B
    lengths = _lengths(doc_lengths, B, Ld, D.device)
    if K == 0:
        return torch.zeros(B, device=D.device, dtype=torch.float32)
    if Ld == 0:
        return torch.full((B,), float("-inf"), device=D.device, dtype=torch.float32)
    assert Lq >= 1
    Qh = _half(Q)
    Dh = _half(D)
    idx = indices.to(torch.int32).contiguous()
    scores = torch.empty(B, device=D.device, dtype=torch.float32)
    if B == 0:
        return scores
    dev = D.device
    _before_call(dev)
    with _lib.on_device(dev):
        rc = lib.fm_maxsim_sparse_fwd(Qh.data_ptr(), Dh.data_ptr(), idx.data_ptr(),
                                      _lib.ptr(lengths), scores.data_ptr(), B, K, Lq, Ld,
                                      Qh.shape[-1], _lib.status_word(dev).data_ptr(),
                                      _lib.stream_of(dev))
    _lib.check(rc, "fm_maxsim_sparse_fwd")
    _after_call(dev)
    return scores


def maxsim_sparse_naive(Q: torch.Tensor, D: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """Reference sparse MaxSim (flash_maxsim/flash_maxsim_sparse.py:143-157).
    Q: [Lq, d], D: [B, Ld, d], indices: [B, K] -> [B] (no length masking)."""
    q_sel = Q[indices.long()]
    sim = torch.einsum("bkd,bld->bkl", q_sel.float(), D.float())
    return sim.max(dim=2).values.sum(dim=1)
