"""Per-device decode workspace.

The reference allocates its logits and segment buffers with torch on every call
(paged_decode.py:179, 206; paged_quant.py:251, 379, 401). Here one workspace per
device is kept and grown only when a call needs more, so steady-state decode
allocates nothing and the same pointer is reused inside captured CUDA graphs.
Call ``reserve()`` with the largest shapes before capturing a graph.
"""
from __future__ import annotations

import torch

from . import _lib

_ws: dict[int, torch.Tensor] = {}


def bytes_needed(n: int, num_heads: int, num_kv_heads: int, k_width: int, v_rank: int, max_seq_len: int) -> int:
    return int(_lib.lib().starkv_decode_workspace_bytes(n, num_heads, num_kv_heads, k_width, v_rank, max_seq_len))


def get(device: torch.device, nbytes: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _ws.get(idx)
    if ws is None or ws.numel() < nbytes:
        # 256-byte alignment is guaranteed by the caching allocator
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        _ws[idx] = ws
    return ws


def reserve(device: torch.device, n: int, num_heads: int, num_kv_heads: int, k_width: int, v_rank: int,
            max_seq_len: int) -> torch.Tensor:
    return get(device, bytes_needed(n, num_heads, num_kv_heads, k_width, v_rank, max_seq_len))


def read_status(ws: torch.Tensor, reset: bool = True) -> int:
    """Device status word of a workspace (synchronises; tests / debugging only)."""
    import ctypes as C
    out = C.c_int32(0)
    st = _lib.lib().starkv_read_status(ws.data_ptr(), C.byref(out), int(reset), _lib.stream_ptr(ws.device))
    _lib.check(st, "starkv_read_status")
    return int(out.value)
