"""The allocation-free decode entry point, called through the C ABI.

starkv_paged_decode_bf16_noalloc is for callers that cannot allocate device
memory (their device memory is all handed out up front, or an engine hosting
this library owns every allocation): it runs in a scratch array built into the
library instead of a caller workspace. These tests check that two calls in a
row agree with the workspace entry point (starkv_paged_decode_bf16) on the same
inputs, within the decode tolerance used everywhere else (2e-2 abs + 1e-2 rel),
that a call too large for the built-in scratch is refused before any GPU work,
and that device-side errors recorded in the built-in scratch reach the caller
through starkv_noalloc_read_status. The workspace entry point is the reference
here because its own tests pin it to the oracle (tests/test_gpu_decode.py);
agreeing with it within the tolerance is agreeing with the oracle. This file
is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _args(layer, out):
    from starkv_b200 import _lib
    a = _lib.DecodeArgs()
    q, kv, bt = layer.query, layer.kv_cache, layer.block_table
    a.query, a.q_stride, a.q_dtype = q.data_ptr(), _lib.i64s(q.stride()), _lib.dtype_code(q)
    a.kv_cache, a.cache_stride, a.cache_dtype = kv.data_ptr(), _lib.i64s(kv.stride()), _lib.dtype_code(kv)
    a.num_blocks, a.block_size = kv.shape[0], kv.shape[1]
    a.block_table, a.bt_stride, a.max_blocks = bt.data_ptr(), _lib.i64s(bt.stride()), bt.shape[1]
    a.seq_lens = layer.seq_lens.data_ptr()
    a.n, a.num_heads, a.num_kv_heads, a.head_dim = q.shape[0], q.shape[1], len(layer.ranks), q.shape[2]
    a.max_seq_len = layer.max_seq_len
    a.k_up, a.k_up_stride, a.k_up_dtype = layer.k_up.data_ptr(), _lib.i64s(layer.k_up.stride()), \
        _lib.dtype_code(layer.k_up)
    a.k_ranks, a.k_head_offsets, a.k_width = layer.k_ranks.data_ptr(), layer.k_head_offsets.data_ptr(), layer.k_width
    vu = layer.v_up_by_q
    a.v_up_by_q, a.v_up_stride, a.v_up_dtype = vu.data_ptr(), _lib.i64s(vu.stride()), _lib.dtype_code(vu)
    a.v_rank = layer.v_rank
    cs = layer.cos_sin_cache
    a.cos_sin_cache, a.cs_stride, a.cs_dtype, a.cs_rows = cs.data_ptr(), _lib.i64s(cs.stride()), \
        _lib.dtype_code(cs), cs.shape[0]
    a.scale = float(layer.scale)
    a.out, a.out_stride, a.out_dtype = out.data_ptr(), _lib.i64s(out.stride()), _lib.dtype_code(out)
    return a


def _close(got, ref):
    got, ref = got.float().cpu().numpy(), ref.float().cpu().numpy()
    err = np.abs(got - ref)
    assert np.all(err <= ATOL + RTOL * np.abs(ref)), f"max abs err {err.max():.3e}"


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from starkv_b200 import _lib
    from starkv_b200.kernels.paged_decode import paged_starkv_decode
    from starkv_b200.workload import make_layer
    dev = torch.device("cuda", 0)
    lib = _lib.lib()
    # two different batches, called back to back on the same stream
    layers = [make_layer([300, 17, 1000, 64], num_heads=32, seed=21, device=dev),
              make_layer([1, 129, 2048], num_heads=32, seed=22, device=dev)]
    for layer in layers:
        need = lib.starkv_decode_workspace_bytes(layer.n, 32, 32, layer.k_width, layer.v_rank, layer.max_seq_len)
        assert need <= 16 << 20
        ref = paged_starkv_decode(layer.query, layer.kv_cache, layer.block_table, layer.seq_lens, layer.max_seq_len,
                                  layer.k_up, layer.k_ranks, layer.k_head_offsets, layer.k_width, layer.v_up_by_q,
                                  layer.cos_sin_cache, layer.scale)
        out = torch.full_like(ref, float("nan"))
        st = lib.starkv_paged_decode_bf16_noalloc(_args(layer, out), _lib.stream_ptr(dev))
        assert st == 0, lib.starkv_strerror(st)
        torch.cuda.synchronize()
        _close(out, ref)


def test_noalloc_refuses_calls_larger_than_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from starkv_b200 import _lib
    from starkv_b200.workload import make_layer
    dev = torch.device("cuda", 0)
    lib = _lib.lib()
    layer = make_layer([40], num_heads=32, seed=23, device=dev)
    out = torch.zeros(1, 32, 128, dtype=torch.bfloat16, device=dev)
    a = _args(layer, out)
    a.n, a.max_seq_len = 64, 8192   # config-2 batch: ~70 MB of scratch, refused before any GPU work
    assert lib.starkv_decode_workspace_bytes(64, 32, 32, layer.k_width, layer.v_rank, 8192) > 16 << 20
    st = lib.starkv_paged_decode_bf16_noalloc(a, _lib.stream_ptr(dev))
    assert st == 102   # STARKV_EWORKSPACE
    assert not out.any()


def test_noalloc_reports_device_errors_through_its_status_word():
    """A block id outside the cache is skipped by the kernels and recorded in the
    built-in scratch's status word; the caller reads it with
    starkv_noalloc_read_status, and the next call starts from a clear word."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from starkv_b200 import _lib
    from starkv_b200.workload import make_layer
    dev = torch.device("cuda", 0)
    lib = _lib.lib()
    layer = make_layer([40, 40], num_heads=32, seed=24, device=dev)
    good_bt = layer.block_table
    layer.block_table = good_bt.clone()
    layer.block_table[1, 1] = layer.kv_cache.shape[0] + 1000   # outside the cache
    out = torch.zeros(layer.n, 32, 128, dtype=torch.bfloat16, device=dev)
    st = lib.starkv_paged_decode_bf16_noalloc(_args(layer, out), _lib.stream_ptr(dev))
    assert st == 0, lib.starkv_strerror(st)
    word = _lib.i32(0)
    assert lib.starkv_noalloc_read_status(C.byref(word), 0, _lib.stream_ptr(dev)) == 0
    assert word.value == 105   # STARKV_EBOUNDS
    layer.block_table = good_bt
    st = lib.starkv_paged_decode_bf16_noalloc(_args(layer, out), _lib.stream_ptr(dev))
    assert st == 0, lib.starkv_strerror(st)
    assert lib.starkv_noalloc_read_status(C.byref(word), 1, _lib.stream_ptr(dev)) == 0
    assert word.value == 0
