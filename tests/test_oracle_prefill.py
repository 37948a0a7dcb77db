"""CPU checks of the oracle's restatements for the dense prefill's attention
(attention.py:246-250) and the step's code rows (model.py:70): against torch's own
CPU attention and matmul in float64."""
import numpy as np
import torch

import starkv_oracle as O


def torch_causal(q, k, v, lens, scale):
    qt, kt, vt = (torch.from_numpy(a) for a in (q, k, v))
    H = q.shape[1]
    out, s0 = [], 0
    for L in lens:
        qs = qt[s0:s0 + L].transpose(0, 1)
        ks = kt[s0:s0 + L].transpose(0, 1).repeat_interleave(H // k.shape[1], dim=0)
        vs = vt[s0:s0 + L].transpose(0, 1).repeat_interleave(H // v.shape[1], dim=0)
        out.append(torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=scale)
                   .transpose(0, 1))
        s0 += L
    return torch.cat(out).numpy()


def test_causal_attention_matches_torch_mha_and_gqa():
    rng = np.random.default_rng(0)
    lens = [1, 7, 33]
    T = sum(lens)
    for hk, hv in ((4, 4), (2, 4), (1, 1)):
        q = rng.standard_normal((T, 4, 128))
        k = rng.standard_normal((T, hk, 128))
        v = rng.standard_normal((T, hv, 128))
        got = O.causal_attention(q, k, v, lens, 0.09)
        assert np.abs(got - torch_causal(q, k, v, lens, 0.09)).max() < 1e-12


def test_causal_attention_first_query_sees_only_itself():
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((5, 2, 128)) for _ in range(3))
    out = O.causal_attention(q, k, v, [5], 1.0)
    assert np.allclose(out[0], v[0])


def test_code_rows_are_the_down_projection():
    rng = np.random.default_rng(2)
    x, w = rng.standard_normal((3, 64)), rng.standard_normal((10, 64))
    assert np.allclose(O.code_rows(x, w), torch.nn.functional.linear(torch.from_numpy(x), torch.from_numpy(w)).numpy())
