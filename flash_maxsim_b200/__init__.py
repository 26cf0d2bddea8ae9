"""flash_maxsim_b200 -- MaxSim (ColBERT / ColPali late-interaction) scoring on
NVIDIA B200, written for sm_100a: TMA-fed tcgen05 tensor-core kernels with
the row-max / sum epilogue fused in TMEM, behind the flash_maxsim 0.1.0 API.

    from flash_maxsim_b200 import flash_maxsim, flash_maxsim_batched
"""
__version__ = "0.1.0"

from ._lib import check_status, LOADED_PATH  # noqa: F401  (loads the CUDA library)
from .api import (  # noqa: F401
    flash_maxsim,
    flash_maxsim_batched,
    flash_maxsim_batched_from_host,
    flash_maxsim_topk,
    flash_maxsim_batched_topk,
    flash_maxsim_packed,
    pack_documents,
    topk_scores,
    flash_maxsim_train,
    maxsim_naive,
    flash_maxsim_int8,
    quantize_int8,
    dequantize_int8,
    flash_maxsim_fp8,
    quantize_fp8,
    dequantize_fp8,
    flash_maxsim_sparse,
    maxsim_sparse_naive,
)

__all__ = [
    "flash_maxsim",
    "flash_maxsim_batched",
    "flash_maxsim_batched_from_host",
    "flash_maxsim_topk",
    "flash_maxsim_batched_topk",
    "flash_maxsim_packed",
    "pack_documents",
    "topk_scores",
    "flash_maxsim_train",
    "maxsim_naive",
    "flash_maxsim_int8",
    "quantize_int8",
    "dequantize_int8",
    "flash_maxsim_fp8",
    "quantize_fp8",
    "dequantize_fp8",
    "flash_maxsim_sparse",
    "maxsim_sparse_naive",
    "check_status",
]
