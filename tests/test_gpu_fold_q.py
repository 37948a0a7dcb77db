"""GPU parity of the exported fold_q operator (paged_quant.py:223-255) against the
oracle restatement and the reference's own output (tests/golden/fold_q.npz, made
by the reference's Triton kernel under its CPU interpreter).

Tolerance: the result is float16; each element within one float16 ulp of the
expected value (the kernels may fuse one multiply-add differently), and almost
all bit-equal.
"""
import os

import numpy as np
import pytest
import torch

import starkv_oracle as O

pytestmark = pytest.mark.gpu


def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def bf16(bits, dev):
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def assert_within_ulp(got, ref):
    got = np.asarray(got, np.float32)
    ref16 = np.asarray(ref, np.float16)
    d = np.abs(got - ref16.astype(np.float32))
    ulp = np.spacing(np.abs(ref16)).astype(np.float32)
    assert np.all(d <= ulp), f"max diff {d.max():.3e}"
    assert (d == 0).mean() > 0.99


def test_fold_q_matches_reference_fixture(golden_dir):
    from starkv_b200.kernels import paged_quant as pq
    dev = cuda()
    c = dict(np.load(os.path.join(golden_dir, "fold_q.npz")))
    q, k_up = bf16(c["query"], dev), bf16(c["k_up"], dev)
    hol = torch.from_numpy(c["head_of_lane"]).to(dev)
    ab = pq.fold_q(q, k_up, hol, float(c["scale"]))
    assert ab.dtype == torch.float16 and ab.shape == c["ab_f16"].shape
    assert_within_ulp(ab.float().cpu().numpy(), c["ab_f16"])


@pytest.mark.parametrize("qdt,udt", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float32),
                                     (torch.float32, torch.bfloat16)])
def test_fold_q_matches_oracle_config_geometry(qdt, udt):
    """32 heads at the config ranks, 64 sequences, mixed input dtypes."""
    from starkv_b200.kernels import paged_quant as pq
    from starkv_b200.workload import sample_ranks
    dev = cuda()
    ranks, _ = sample_ranks(32, 0)
    _, offsets, W = O.k_layout(ranks)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(64, 32, 128, generator=g).to(qdt)
    k_up = torch.zeros(W, 128)
    for r, o in zip(ranks, offsets):
        k_up[o:o + r] = torch.randn(r, 128, generator=g) / r ** 0.5
    k_up = k_up.to(udt)
    _, hol, _ = pq.k_tables(ranks, dev)
    ab = pq.fold_q(q.to(dev), k_up.to(dev), hol, 128 ** -0.5)
    ref = O.fold_q(q.float().numpy(), k_up.float().numpy(), hol.cpu().numpy(), 128 ** -0.5)
    assert_within_ulp(ab.float().cpu().numpy(), ref)


def test_fold_q_records_out_of_range_head():
    """A head_of_lane entry outside [0, H) is recorded as EBOUNDS in the status
    word and its row is zero; the other rows are unchanged."""
    from starkv_b200.kernels import paged_quant as pq
    dev = cuda()
    ranks = [16, 32]
    _, offsets, W = O.k_layout(ranks)
    g = torch.Generator().manual_seed(6)
    q = torch.randn(2, 2, 128, generator=g).to(torch.bfloat16).to(dev)
    k_up = torch.randn(W, 128, generator=g).to(torch.bfloat16).to(dev)
    _, hol, _ = pq.k_tables(ranks, dev)
    good = pq.fold_q(q, k_up, hol, 0.1)
    bad_hol = hol.clone()
    bad_hol[3] = 7
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ab = pq.fold_q(q, k_up, bad_hol, 0.1, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 105
    assert not ab[:, 3].any()
    keep = torch.ones(W, dtype=torch.bool, device=dev)
    keep[3] = False
    assert torch.equal(ab[:, keep], good[:, keep])
