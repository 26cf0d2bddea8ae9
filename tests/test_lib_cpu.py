"""Host-side checks that need no GPU: the C-ABI library loads and exports
every entry point include/flash_maxsim_sm100.h declares, argument errors
come back as codes, plans exist for every BASELINE configuration, and the
Python API refuses non-CUDA tensors (there is no CPU path)."""
import re

import pytest
import torch

from tests.conftest import ROOT

HEADER = ROOT / "include" / "flash_maxsim_sm100.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(fm_\w+)\s*\(", text, flags=re.M)))


def test_exports_every_declared_symbol():
    from flash_maxsim_b200 import _lib
    names = declared_functions()
    assert len(names) >= 9, names
    for n in names:
        assert hasattr(_lib.lib, n), n
        assert n in _lib.SIGNATURES, f"{n} declared in the header but not bound"


def test_status_strings_and_version():
    from flash_maxsim_b200 import _lib
    assert _lib.lib.fm_abi_version() >= 100
    for code in (0, 1, 2, 10, 14, 18, 19, 20, 21, 22):
        assert _lib.status_string(code) != "unknown status"
    assert _lib.status_string(9999) == "unknown status"


def test_argument_errors_without_device():
    from flash_maxsim_b200 import _lib
    L = _lib.lib
    assert L.fm_maxsim_fwd(None, None, None, None, None, 1, 1, 32, 300, 128, 1, None, None) == _lib.FM_ERR_ARG
    assert L.fm_maxsim_int8_fwd(None, None, None, None, None, None, 1, 32, 300, 128, None, None) == _lib.FM_ERR_ARG
    assert L.fm_maxsim_sparse_fwd(None, None, None, None, None, 1, 4, 32, 300, 128, None, None) == _lib.FM_ERR_ARG
    assert L.fm_maxsim_bwd(None, None, None, None, None, None, 1, 1, 32, 300, 128, None, 0, None) == _lib.FM_ERR_ARG
    assert L.fm_maxsim_bwd_workspace_size(64, 4096, 64, 1024, 256) > 0
    assert L.fm_quantize_int8(None, 0, None, None, None, 10, 128, None) == _lib.FM_ERR_ARG
    assert L.fm_wait_selftest(None, 1000, None) == _lib.FM_ERR_ARG


@pytest.mark.parametrize("args", [
    (0, False, 1, 1000, 32, 300, 128),        # config 1
    (0, False, 100, 100000, 32, 300, 128),    # config 2
    (0, False, 16, 4000, 1024, 1024, 128),    # config 3
    (2, False, 1, 200000, 32, 300, 128),      # config 4
    (0, True, 64, 4096, 64, 1024, 256),       # config 5 (forward with argmax)
    (1, False, 1, 50, 32, 300, 128),          # sparse
    (0, False, 1, 20, 32, 128, 2048),         # largest embedding dim
])
def test_plans_fit_shared_memory(args):
    from flash_maxsim_b200._lib import plan_info
    p = plan_info(*args)
    assert 120 * 1024 <= p["smem"] <= 232448
    assert p["C"] % 16 == 0 and 16 <= p["C"] <= 256
    assert p["ts_stride"] * p["nts"] <= 512 and p["nts"] >= 1
    assert p["nd"] >= p["G"] >= 1
    if p["nk"] > 1:
        assert p["G"] <= p["nts"]


def test_plan_even_tmem_slots_for_two_issuers():
    """Config-2 shapes: 192-token chunks (2 TMEM slots, one per MMA issuer)
    rather than 160 (3 slots); MMAs with N <= 192 cost the same."""
    from flash_maxsim_b200._lib import plan_info
    p = plan_info(0, False, 100, 100000, 32, 300, 128)
    assert p["C"] == 192 and p["nts"] == 2
    for args in [(0, False, 16, 4000, 1024, 1024, 128), (0, False, 8, 100, 32, 300, 128), (0, True, 3, 40, 64, 200, 128)]:
        q = plan_info(*args)
        assert q["nts"] >= 2 and q["ts_stride"] * q["nts"] <= 512


def test_plan_groups_short_documents():
    from flash_maxsim_b200._lib import plan_info
    assert plan_info(0, False, 100, 100000, 32, 128, 128)["gd"] >= 2
    assert plan_info(0, False, 16, 4000, 1024, 1024, 128)["gd"] == 1
    assert plan_info(0, False, 1, 1000, 32, 300, 128)["q_resident"] == 1


def test_api_rejects_cpu_tensors():
    import flash_maxsim_b200 as fm
    Q = torch.randn(32, 128)
    D = torch.randn(2, 10, 128)
    with pytest.raises(ValueError, match="CUDA"):
        fm.flash_maxsim(Q, D)
    with pytest.raises(ValueError, match="CUDA"):
        fm.quantize_int8(D)
    with pytest.raises(AssertionError):
        fm.flash_maxsim(Q, torch.randn(2, 10, 64))


def test_reference_helpers_are_plain_torch():
    # maxsim_naive / maxsim_sparse_naive / dequantize_int8 are the reference's
    # own torch helpers and keep working on any device
    import flash_maxsim_b200 as fm
    from oracle import maxsim_oracle as O
    Q, D = O.seeded_inputs(0, (8, 16), (3, 5, 16))
    got = fm.maxsim_naive(torch.from_numpy(Q), torch.from_numpy(D)).numpy()
    assert abs(got - O.maxsim(Q, D)).max() < 1e-4


def test_host_streaming_pieces_cover_the_corpus():
    # flash_maxsim_batched_from_host's piece plan: contiguous, disjoint,
    # covering [0, B), each piece within the byte budget unless one document
    # alone exceeds it
    from flash_maxsim_b200.api import host_pieces
    for B, doc, budget in [(100000, 300 * 128 * 2, 512 << 20), (3000, 76800, 10 << 20), (7, 10, 1),
                           (1, 1 << 30, 512 << 20), (5, 100, 1000), (0, 100, 1000)]:
        piece, n = host_pieces(B, doc, budget)
        assert piece >= 1
        spans = [(i * piece, min(B, (i + 1) * piece)) for i in range(n)]
        covered = [b for lo, hi in spans for b in range(lo, hi)] if B <= 10000 else None
        if covered is not None:
            assert covered == list(range(B))
        assert all(hi > lo for lo, hi in spans)
        assert piece * doc <= budget or piece == 1
        assert n == (0 if B == 0 else -(-B // piece))
