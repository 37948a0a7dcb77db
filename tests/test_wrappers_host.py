"""CPU checks of the Python operators that front the prefill attention and the fused
K/V down-projection + cache write: their argument checks refuse bad calls before any
library call, and the prompt bookkeeping (cu_seqlens, query tiles) is right."""
import pytest
import torch

from starkv_b200.kernels import paged_decode as pd
from starkv_b200.kernels import prefill as pf


def test_cu_seqlens_are_prompt_offsets():
    cu = pf.cu_seqlens_of([5, 128, 0, 300], "cpu")
    assert cu.dtype == torch.int32
    assert cu.tolist() == [0, 5, 133, 133, 433]


@pytest.mark.parametrize("case", ["head_dim", "tokens", "lens", "dtype", "mixed", "stride"])
def test_prefill_attention_refuses_bad_arguments(case):
    T, H = 10, 4
    q = torch.zeros(T, H, 128, dtype=torch.bfloat16)
    k = torch.zeros(T, 2, 128, dtype=torch.bfloat16)
    v = torch.zeros(T, H, 128, dtype=torch.bfloat16)
    lens = [4, 6]
    if case == "head_dim":
        q = torch.zeros(T, H, 64, dtype=torch.bfloat16)
    elif case == "tokens":
        k = torch.zeros(T + 1, 2, 128, dtype=torch.bfloat16)
    elif case == "lens":
        lens = [4, 5]
    elif case == "dtype":
        q, k, v = q.float(), k.float(), v.float()
    elif case == "mixed":
        v = v.half()
    elif case == "stride":
        q = torch.zeros(T, H, 256, dtype=torch.bfloat16)[:, :, ::2]
    with pytest.raises(ValueError):
        pf.prefill_attention(q, k, v, lens, 0.1)


def test_prefill_attention_empty_needs_no_library():
    out = pf.prefill_attention(torch.zeros(0, 2, 128, dtype=torch.bfloat16), torch.zeros(0, 1, 128, dtype=torch.bfloat16),
                               torch.zeros(0, 2, 128, dtype=torch.bfloat16), [], 0.1)
    assert out.shape == (0, 2, 128)


def test_kv_down_write_refuses_bad_arguments():
    cache = torch.zeros(4, 16, 96, dtype=torch.bfloat16)
    slots = torch.zeros(3, dtype=torch.int32)
    x = torch.zeros(3, 512, dtype=torch.bfloat16)
    w = torch.zeros(96, 512, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        pd.kv_down_write(x.half(), w, cache, slots)          # hidden not in the cache dtype
    with pytest.raises(ValueError):
        pd.kv_down_write(x, w.float(), cache, slots)         # weights not in the cache dtype
    with pytest.raises(ValueError):
        pd.kv_down_write(torch.zeros(3, 1024, dtype=torch.bfloat16)[:, ::2], w, cache, slots)   # strided rows
    pd.kv_down_write(x[:0], w, cache, slots[:0])             # nothing to write: no library call
