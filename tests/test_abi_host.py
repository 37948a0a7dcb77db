"""CPU checks of the boundary and the host logic (no GPU work is launched).

* the C-ABI library loads and exports every entry point that include/starkv_b200.h
  declares, and its struct layouts match the ctypes binding;
* host-side argument checks return their error codes before touching a GPU;
* the Python mirrors of the reference's format helpers (paged_quant.py:46-131)
  agree with the CPU oracle;
* head sharding deals equal head counts with balanced K width.
"""
import ctypes as C
import os
import re

import numpy as np
import pytest
import torch

import starkv_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "starkv_b200.h")


@pytest.fixture(scope="module")
def lib():
    import importlib.util
    spec = importlib.util.spec_from_file_location("starkv_build", os.path.join(ROOT, "star-kv-serve_b200", "build.py"))
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    build.build()            # no-op when the library is up to date
    from starkv_b200 import _lib
    return _lib.lib()


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"STARKV_API\s+[\w\s\*]+?\b(starkv_\w+)\s*\(", text)


def test_header_declares_the_entry_points():
    names = declared_symbols()
    for must in ("starkv_paged_decode_bf16", "starkv_paged_decode_q32", "starkv_pack_kv_q32",
                 "starkv_fold_q", "starkv_decode_workspace_bytes", "starkv_paged_decode_bf16_noalloc"):
        assert must in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol(lib):
    from starkv_b200 import _lib
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    # the binding knows every declared entry point, and the struct layouts agree
    assert set(declared_symbols()) <= set(_lib.EXPORTS) | {"starkv_version", "starkv_strerror"}
    _lib.check_abi()


def test_version_and_error_strings(lib):
    lib.starkv_version.restype = C.c_char_p
    lib.starkv_strerror.restype = C.c_char_p
    assert lib.starkv_version().decode()
    for code in (0, 22, 100, 101, 102, 103, 104, 105, 106):
        assert lib.starkv_strerror(code).decode()


def test_workspace_size_is_host_arithmetic(lib):
    n, H, W, rv, L = 64, 32, 1392, 1536, 8192
    need = lib.starkv_decode_workspace_bytes(n, H, H, W, rv, L)
    # AB image + rotary tiles + e16 + tile maxima + sums + pv, all 256-aligned
    lower = n * ((W + 127) // 128) * 128 * 256 + L * 256 + n * H * L * 2 + n * H * (L // 128) * 4 + n * H * rv * 4
    assert lower <= need <= lower + 64 * 1024
    assert lib.starkv_decode_workspace_bytes(-1, H, H, W, rv, L) == 0
    assert lib.starkv_decode_workspace_bytes(n, 0, H, W, rv, L) == 0


def test_entry_points_reject_bad_arguments_before_any_gpu_work(lib):
    from starkv_b200 import _lib
    assert lib.starkv_paged_decode_bf16(None, None, 0, None) == 22
    assert lib.starkv_paged_decode_q32(None, None, 0, None) == 22
    assert lib.starkv_paged_decode_bf16_noalloc(None, None) == 22
    assert lib.starkv_pack_kv_q32(None, None) == 22
    a = _lib.DecodeArgs()
    a.n, a.num_heads, a.num_kv_heads, a.k_width, a.v_rank, a.max_seq_len = 64, 32, 32, 1392, 1536, 8192
    assert lib.starkv_paged_decode_bf16_noalloc(C.byref(a), None) == 102   # larger than its scratch
    assert lib.starkv_noalloc_read_status(None, 0, None) == 22
    # fold_q: element types and the lane count are checked before any GPU work
    qs, us = _lib.i64s([4096, 128, 1]), _lib.i64s([128, 1])
    fake = C.c_void_p(4096)   # never dereferenced: every call below is refused first
    assert lib.starkv_fold_q(fake, qs, _lib.U8, fake, us, _lib.BF16, fake, 2, 32, 64, 0.1, fake, None, None) == 101
    assert lib.starkv_fold_q(fake, qs, _lib.BF16, fake, us, 9, fake, 2, 32, 64, 0.1, fake, None, None) == 101
    assert lib.starkv_fold_q(fake, qs, _lib.BF16, fake, us, _lib.BF16, fake, 2, 32, 40, 0.1, fake, None, None) == 22
    assert lib.starkv_fold_q(None, qs, _lib.BF16, fake, us, _lib.BF16, fake, 2, 32, 64, 0.1, fake, None, None) == 22
    # prefill attention: pointers, head counts, dtype and alignment are checked first
    s2 = _lib.i64s([4096, 128])
    pa = lambda q, dt, H, Hk, Hv, st=s2: lib.starkv_prefill_attention(  # noqa: E731
        q, st, fake, s2, fake, s2, dt, 100, H, Hk, Hv, fake, 2, 1, 0.1, fake, s2, None, None)
    assert pa(None, _lib.BF16, 32, 8, 32) == 22
    assert pa(fake, _lib.BF16, 32, 5, 32) == 22          # 32 query heads over 5 K heads
    assert pa(fake, _lib.F32, 32, 8, 32) == 101
    assert pa(fake, _lib.BF16, 32, 8, 32, _lib.i64s([4100, 128])) == 100   # row stride not 16-byte aligned
    # fused K/V down-projection + cache write: shapes, dtype and alignment first
    cs = _lib.i64s([16 * 2928, 2928])
    kd = lambda h, dt, hid, st=cs, hs=4096: lib.starkv_kv_down_cache_write(  # noqa: E731
        h, hs, fake, 4096, dt, 64, hid, 2928, fake, st, 64, 16, fake, _lib.I32, None, None)
    assert kd(None, _lib.BF16, 4096) == 22
    assert kd(fake, _lib.BF16, 4000) == 22                 # hidden not a multiple of 512
    assert kd(fake, _lib.F32, 4096) == 101
    assert kd(fake, _lib.BF16, 4096, _lib.i64s([16 * 2928, 2000])) == 22    # cache row narrower than the codes
    assert kd(fake, _lib.BF16, 4096, hs=4100) == 100        # hidden row stride not 16-byte aligned


def test_quant_row_matches_oracle():
    from starkv_b200.kernels import paged_quant as pq
    for ranks, rv in (([16, 32, 48, 64], 192), ([16] * 8, 32), ([64, 64, 16, 32, 48, 16], 1536), ([160, 32], 96)):
        _, _, W = O.k_layout(ranks)
        mine, ref = pq.QuantRow(W, len(ranks), rv), O.QuantRow(W, len(ranks), rv)
        for f in ("ks_off", "vs_off", "vq_off", "v_nout", "v_nbo", "v_bytes", "nbytes"):
            assert getattr(mine, f) == getattr(ref, f), (ranks, rv, f)


def test_k_tables_match_oracle():
    from starkv_b200.kernels import paged_quant as pq
    for ranks in ([16, 32, 48, 64], [64, 16, 160, 32], [16] * 5):
        head_of_lane, nouts, tiles = pq.k_tables(ranks, "cpu")
        ref = O.k_tables(ranks)
        np.testing.assert_array_equal(head_of_lane.numpy(), ref[0])
        np.testing.assert_array_equal(nouts.numpy(), ref[1])
        for t, r in zip(tiles, ref[2]):
            np.testing.assert_array_equal(t.numpy(), r)


def test_n_outlier_and_block_hadamard_match_oracle():
    from starkv_b200.kernels import paged_quant as pq
    for r in (16, 32, 48, 64, 128, 1536):
        assert pq.n_outlier(r) == O.n_outlier(r)
        g1 = torch.Generator().manual_seed(pq.HADAMARD_SEED)
        g2 = torch.Generator().manual_seed(pq.HADAMARD_SEED)
        a = pq.block_hadamard(r, pq.n_outlier(r), g1).numpy()
        b = O.block_hadamard(r, O.n_outlier(r), g2)
        np.testing.assert_array_equal(a, b)
        np.testing.assert_allclose(a @ a.T, np.eye(r), atol=1e-12)


def test_lpt_shard_equal_counts_and_balanced_width():
    from starkv_b200.sharding import align16, lpt_shard, shard_lanes, shard_loads
    from starkv_b200.workload import sample_ranks
    for seed, skew in ((0, False), (1, True), (7, True)):
        ranks, _ = sample_ranks(32, seed, skew)
        for world in (1, 2, 4, 8):
            groups = lpt_shard(ranks, world)
            assert sorted(h for g in groups for h in g) == list(range(32))
            assert all(len(g) == 32 // world for g in groups)
            loads = shard_loads(ranks, groups)
            assert max(loads) - min(loads) <= max(align16(r) for r in ranks)
            assert groups == lpt_shard(ranks, world)   # deterministic
            for g in groups:
                lr, lo, lw, lanes = shard_lanes(ranks, g)
                assert lw == sum(align16(r) for r in lr) and len(lanes) == lw
                assert lo == O.k_layout(lr)[1]
    with pytest.raises(ValueError):
        lpt_shard([16] * 30, 4)
