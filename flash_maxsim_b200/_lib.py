"""ctypes binding of libflashmaxsim_sm100.so (C ABI: include/flash_maxsim_sm100.h).

The library must exist: importing this module without it raises ImportError.
There is no fallback implementation.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
from pathlib import Path

import torch

from .build import LIB_PATH

FM_OK = 0
FM_ERR_ARG = 1
FM_ERR_LAUNCH = 2
FM_ERR_TIMEOUT_SELFTEST = 19
FM_ERR_BAD_INDEX = 20
FM_ERR_UNSUPPORTED = 21
FM_ERR_SCRATCH_TOO_SMALL = 23
FM_DTYPE_F16 = 0
FM_OPT_FLAT_KERNEL = 1
FM_DTYPE_F32 = 1
FM_DTYPE_BF16 = 2

# exported symbol -> (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
SIGNATURES = {
    "fm_abi_version": (_I, []),
    "fm_status_string": (ctypes.c_char_p, [_I]),
    "fm_set_wait_timeout_ns": (None, [_I64]),
    "fm_set_option": (_I, [_I, _I]),
    "fm_maxsim_fwd": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "fm_maxsim_packed_fwd": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I64, _P, _P]),
    "fm_maxsim_int8_fwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "fm_maxsim_sparse_fwd": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "fm_maxsim_bwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I64, _P]),
    "fm_maxsim_bwd_workspace_size": (_I64, [_I, _I, _I, _I, _I]),
    "fm_maxsim_bwd_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "fm_maxsim_fp8_fwd": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "fm_quantize_fp8": (_I, [_P, _I, _P, _P, _I64, _I, _P]),
    "fm_normalize_quantize_int8": (_I, [_P, _I, _P, _P, _P, _I64, _I, _P]),
    "fm_normalize_quantize_fp8": (_I, [_P, _I, _P, _P, _I64, _I, _P]),
    "fm_quantize_int8": (_I, [_P, _I, _P, _P, _P, _I64, _I, _P]),
    "fm_wait_selftest": (_I, [_P, _I64, _P]),
    "fm_fwd_plan_info": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, _I, _P, _I]),
    "fm_topk_workspace_size": (_I64, [_I, _I]),
    "fm_maxsim_topk": (_I, [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _P, _I64, _P, _P]),
    "fm_topk_select": (_I, [_P, _I, _I, _I, _I64, _P, _P, _P, _I64, _P]),
    "fm_topk_merge": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
}

PLAN_FIELDS = ("C", "G", "nd", "nq", "nu", "nk", "kq_atoms", "d_atoms", "RS", "rep",
               "q_resident", "nts", "ts_stride", "smem", "R", "gd")


def plan_info(mode: int, argmax: bool, Nq: int, B: int, Lq: int, Ld: int, d: int,
              shared: bool = True, K: int = 0) -> dict:
    """The forward launch plan for a shape (mode 0 dense, 1 sparse, 2 INT8)."""
    out = (ctypes.c_int32 * len(PLAN_FIELDS))()
    rc = lib.fm_fwd_plan_info(mode, int(argmax), Nq, B, Lq, Ld, d, int(shared), K,
                              ctypes.cast(out, ctypes.c_void_p), len(PLAN_FIELDS))
    check(rc, "fm_fwd_plan_info")
    return dict(zip(PLAN_FIELDS, list(out)))


def set_flat_kernel(enable: bool) -> None:
    """Route eligible shared-document batches to the flat-token kernel
    (process-wide; same scores, different tiling)."""
    check(lib.fm_set_option(FM_OPT_FLAT_KERNEL, int(bool(enable))), "fm_set_option")


def _load() -> ctypes.CDLL:
    path = Path(os.environ.get("FLASH_MAXSIM_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python flash_maxsim_b200/build.py` "
            "(flash_maxsim_b200 has no non-CUDA implementation)"
        )
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()
LOADED_PATH = Path(lib._name)


def status_string(code: int) -> str:
    return lib.fm_status_string(int(code)).decode()


def check(rc: int, what: str) -> None:
    """Raise for a host-side error code returned by an entry point."""
    if rc != FM_OK:
        msg = f"{what}: {status_string(rc)} (code {rc})"
        if rc == FM_ERR_ARG:
            raise ValueError(msg)
        raise RuntimeError(msg)


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device) -> int:
    """Handle of the current CUDA stream of `device` (what kernels launch on)."""
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def on_device(device: torch.device):
    """Context that makes `device` current for a launch (a no-op when it already is)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word that kernels write device-side errors into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def sync_check_enabled() -> bool:
    """FLASH_MAXSIM_SYNC_CHECK=1: synchronise and check after every call."""
    return os.environ.get("FLASH_MAXSIM_SYNC_CHECK", "0") not in ("", "0")


class _Mirror:
    """Pinned host copy of a device's status word, refreshed asynchronously
    after every call; `event` marks when the copy has landed."""

    def __init__(self, device: torch.device):
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.event = torch.cuda.Event()
        self.pending = False


_mirrors: dict[int, _Mirror] = {}


def _raise_device_error(device: torch.device, code: int) -> None:
    status_word(device).zero_()
    raise RuntimeError(f"flash_maxsim_b200 device error: {status_string(code)} (code {code})")


def poll_status(device: torch.device) -> None:
    """Raise RuntimeError if an earlier call on `device` recorded a device-side
    error whose asynchronous copy to the host has landed (no synchronisation)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    m = _mirrors.get(idx)
    if m is None or not m.pending or torch.cuda.is_current_stream_capturing():
        return
    if not m.event.query():
        return
    m.pending = False
    code = int(m.host[0])
    if code != FM_OK:
        m.host.zero_()
        _raise_device_error(torch.device("cuda", idx), code)


def after_call(device: torch.device) -> None:
    """Make device-side errors visible without a synchronisation: the status
    word is copied into pinned host memory behind the call on the current
    stream, and the next call on this device (or check_status) raises when it
    is non-zero. Under stream capture nothing is queued; with
    FLASH_MAXSIM_SYNC_CHECK=1 every call synchronises and checks at once."""
    if sync_check_enabled():
        check_status(device)
        return
    if torch.cuda.is_current_stream_capturing():
        return
    idx = device.index if device.index is not None else torch.cuda.current_device()
    m = _mirrors.get(idx)
    if m is None:
        m = _mirrors[idx] = _Mirror(torch.device("cuda", idx))
    dev = torch.device("cuda", idx)
    with on_device(dev):
        m.host.copy_(status_word(dev), non_blocking=True)
        m.event.record()
    m.pending = True


def check_status(device: torch.device | int | None = None) -> None:
    """Synchronise `device` and raise RuntimeError if a kernel recorded an error.

    Device-side failures (a bounded wait that ran out of time, an index out of
    range) do not abort the CUDA context; they are recorded in the status word
    and reported here. The word is cleared after it has been read.
    """
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    st = status_word(device)
    torch.cuda.synchronize(device)
    m = _mirrors.get(device.index if device.index is not None else torch.cuda.current_device())
    if m is not None:
        m.pending = False
        m.host.zero_()
    code = int(st.item())
    if code != FM_OK:
        _raise_device_error(device, code)
