"""starkv_b200: B200-native (sm_100a) STAR-KV paged low-rank decode attention.

The operator surface mirrors the reference's ``starkv_serve.kernels``:

    from starkv_b200.kernels.paged_decode import paged_starkv_decode
    from starkv_b200.kernels.paged_quant import (paged_quant_decode, pack_kv, fold_q,
        QuantRow, k_tables, n_outlier, block_hadamard)

Everything runs in the C-ABI library ``_lib/libstarkv_b200.so`` (built by
``star-kv-serve_b200/build.py``); there is no CPU or torch fallback.
"""
from ._lib import LIB_PATH, check_abi, lib  # noqa: F401

__version__ = "1.0"
