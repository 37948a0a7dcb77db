"""Pin the CPU oracle to the reference: golden fixtures made by the reference's
own code (tests/golden/make_golden.py) must be reproduced byte-for-byte
(packing, dequantization) and to fp32 rounding (decode math)."""
import glob
import os

import numpy as np
import pytest
import torch

import starkv_oracle as O


def load(golden_dir, name):
    return dict(np.load(os.path.join(golden_dir, name)))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "pack_*.npz"))))
def test_pack_rows_bit_exact(path):
    c = dict(np.load(path))
    ranks = [int(r) for r in c["ranks"]]
    _, _, W = O.k_layout(ranks)
    row = O.QuantRow(W, len(ranks), int(c["v_rank"]))
    assert row.nbytes == int(c["nbytes"])
    k = O.bf16_bits_to_f32(c["k_codes"])
    v = O.bf16_bits_to_f32(c["v_codes"])
    rows = O.pack_rows(k, v, row, ranks)
    np.testing.assert_array_equal(rows, c["rows"])
    kd, vd = O.unpack_rows(rows, row, ranks)
    np.testing.assert_array_equal(kd, c["k_deq"])     # dequantized codes bit-exact
    np.testing.assert_array_equal(vd, c["v_deq"])


def _decode_inputs(c):
    f = O.bf16_bits_to_f32
    return f(c["query"]), f(c["cache"]), f(c["k_up"]), f(c["v_up_by_q"]), f(c["cos_sin"])


@pytest.mark.parametrize("name", ["decode_bf16_mha.npz", "decode_bf16_ragged.npz", "decode_bf16_gqa.npz"])
def test_bf16_decode_matches_reference_math(golden_dir, name):
    c = load(golden_dir, name)
    q, cache, k_up, v_up, cs = _decode_inputs(c)
    out = O.decode_paged_bf16(q, cache, c["block_table"], c["seq_lens"], k_up, c["k_ranks"],
                              c["k_head_offsets"], int(c["k_width"]), v_up, cs, float(c["scale"]))
    np.testing.assert_allclose(out, c["out_ref_fp32"], atol=2e-5, rtol=1e-4)
    # the reference paged Triton kernel (fp16, CPU interpreter) agrees within fp16 noise
    np.testing.assert_allclose(out, c["out_triton_fp16"], atol=5e-3, rtol=5e-3)


@pytest.mark.parametrize("name", ["decode_quant.npz", "decode_quant_b.npz"])
def test_quant_decode_matches_reference_math(golden_dir, name):
    c = load(golden_dir, name)
    f = O.bf16_bits_to_f32
    ranks = [int(r) for r in c["k_ranks"]]
    _, _, W = O.k_layout(ranks)
    row = O.QuantRow(W, len(ranks), int(c["v_rank"]))
    out = O.decode_paged_quant(f(c["query"]), c["cache"], c["block_table"], c["seq_lens"], row, ranks,
                               f(c["k_up"]), f(c["v_up_by_q"]), f(c["cos_sin"]), float(c["scale"]))
    np.testing.assert_allclose(out, c["out_ref_fp32"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(out, c["out_triton_fp16"], atol=1e-2, rtol=1e-2)
    nouts, hol, (th, tn, tl) = O.k_tables(ranks)
    np.testing.assert_array_equal(nouts, c["k_nouts"])
    np.testing.assert_array_equal(hol, c["head_of_lane"])
    np.testing.assert_array_equal(th, c["tile_head"])
    np.testing.assert_array_equal(tn, c["tile_nout"])
    np.testing.assert_array_equal(tl, c["tile_last"])


def test_block_hadamard_matches_reference(golden_dir):
    c = load(golden_dir, "checkpoint_layer.npz")
    for r in (1, 2, 5, 16, 37, 64, 100):
        gen = torch.Generator().manual_seed(O.HADAMARD_SEED)
        T = O.block_hadamard(r, O.n_outlier(r), gen)
        np.testing.assert_array_equal(T, c[f"T{r}"])
        np.testing.assert_allclose(T @ T.T, np.eye(r), atol=1e-12)


def test_quantizer_ties_round_half_even():
    # x/s exactly k+0.5 -> even neighbour (kv_quant.py:111-121 uses torch.round)
    x = np.asarray([[7.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 6.5]], np.float32)
    n, s = O.quantize_block(x, 4)
    assert s[0] == np.float32(1.0)
    np.testing.assert_array_equal(n[0].astype(int) - 8, [7, 0, 2, 2, 0, -2, -2, 6])
    # all-zero block: amax clamps to EPS, every code is 8
    n, s = O.quantize_block(np.zeros((1, 5), np.float32), 3)
    assert s[0] == np.float32(1e-5) / np.float32(3)
    assert (n == 8).all()


def test_fold_q_matches_reference_fixture(golden_dir):
    """The oracle's fold_q against the reference's own fold_q (paged_quant.py:223-255,
    run by Triton's CPU interpreter): equal to within one float16 ulp (the two may
    fuse one multiply-add differently)."""
    c = load(golden_dir, "fold_q.npz")
    f = O.bf16_bits_to_f32
    ab = O.fold_q(f(c["query"]), f(c["k_up"]), c["head_of_lane"], float(c["scale"]))
    ref = c["ab_f16"]
    assert ab.shape == ref.shape
    d = np.abs(ab.astype(np.float32) - ref.astype(np.float32))
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    assert np.all(d <= ulp), f"max diff {d.max()}"
    assert (d == 0).mean() > 0.99
