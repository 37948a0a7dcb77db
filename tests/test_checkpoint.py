"""The fused_weights.pt loader (starkv_b200.checkpoint) against the reference's
own loader: tests/golden/checkpoint_layer.npz holds a small fused state dict and
starkv_serve.checkpoint._load_layer's outputs for it (checkpoint.py:106-169), with
and without kv_quant, made by tests/golden/make_golden.py. The serving layout must
be reproduced bit-exactly (float32). Plus the file-level behaviour of
load_fused_checkpoint (checkpoint.py:74-93) and the layer built from it."""
import numpy as np
import pytest
import torch


def _fixture(golden_dir):
    import os
    c = dict(np.load(os.path.join(golden_dir, "checkpoint_layer.npz")))
    pre = "model.layers.0.self_attn."
    sd = {pre + k[3:]: torch.from_numpy(v) for k, v in c.items() if k.startswith("in_")}
    return c, sd, pre


@pytest.mark.parametrize("quant", [False, True])
def test_load_layer_matches_reference_bit_exact(golden_dir, quant):
    from starkv_b200.checkpoint import load_layer
    c, sd, pre = _fixture(golden_dir)
    lw = load_layer(sd, pre, 0, 4, 128, torch.float32, quant)
    t = "q" if quant else "b"
    for name in ("k_down", "k_up", "v_down", "v_up", "k_head_offsets", "k_head_widths"):
        np.testing.assert_array_equal(getattr(lw, name).numpy(), c[f"{t}_{name}"], err_msg=name)
    assert [lw.k_width, lw.k_max_rank, lw.v_rank, lw.v_rank_real, lw.cache_bytes(2)] == c[f"{t}_meta"].tolist()


def test_load_fused_checkpoint_file(golden_dir, tmp_path):
    """Layers without head ranks are left full-rank; a layer in the unfused format is
    refused; a file without any fused layer is refused."""
    from starkv_b200.checkpoint import load_fused_checkpoint
    c, sd, pre = _fixture(golden_dir)
    moved = {k.replace("layers.0.", "layers.2."): v for k, v in sd.items()}
    p = tmp_path / "fused_weights.pt"
    torch.save({**sd, **moved}, p)
    ck = load_fused_checkpoint(str(p), 4, 4, 128, torch.float32)
    assert sorted(ck.layers) == [0, 2] and ck.skip_layers == (1, 3)
    assert ck.is_compressed(2) and not ck.is_compressed(1)
    np.testing.assert_array_equal(ck.layers[2].k_up.numpy(), c["b_k_up"])
    legacy = {**sd, "model.layers.1.self_attn.k_proj.Sigma_blocks.0.diag": torch.ones(3)}
    torch.save(legacy, p)
    with pytest.raises(ValueError):
        load_fused_checkpoint(str(p), 4, 4, 128)
    torch.save({"model.embed_tokens.weight": torch.zeros(2, 2)}, p)
    with pytest.raises(ValueError):
        load_fused_checkpoint(str(p), 4, 4, 128)
    bad = dict(sd)
    bad[pre + "k_proj.head_ranks"] = torch.tensor([13, 32, 7], dtype=torch.int32)
    with pytest.raises(ValueError):
        load_fused_checkpoint(bad, 1, 4, 128)


@pytest.mark.parametrize("quant", [False, True])
def test_layer_weights_from_checkpoint(quant):
    """A synthetic checkpoint through the loader into the layer's weights: the codes
    times the up-projections equal the checkpoint's U VS products (the Hadamard
    rotation of the 3.2-bit layout cancels), V padded to 16 for bf16 caches, one
    V up-projection per KV head repeated over its query heads."""
    from starkv_b200.checkpoint import load_fused_checkpoint, synthetic_state_dict
    from starkv_b200.layer import AttnWeights
    H, Hd, hidden = 4, 128, 64
    ranks, rv = [13, 32, 7, 40], 50
    sd = synthetic_state_dict({0: (ranks, rv)}, hidden, H, Hd, seed=3, dtype=torch.float32)
    lw = load_fused_checkpoint(sd, 1, H, Hd, torch.float32, kv_quant=quant).layers[0]
    g = torch.Generator().manual_seed(4)
    wq = torch.randn(2 * H * Hd, hidden, generator=g)
    wo = torch.randn(hidden, 2 * H * Hd, generator=g)
    w = AttnWeights.from_checkpoint(lw, wq, wo, num_heads=2 * H, dtype=torch.float32)
    assert w.rotated == quant and w.v_rank == (rv if quant else 64) and w.k_ranks == ranks
    x = torch.randn(5, hidden, generator=g, dtype=torch.float64)
    codes = x @ w.kv_down.double().T
    pre = "model.layers.0.self_attn."
    ku, kvs = sd[pre + "k_proj.U.weight"].double(), sd[pre + "k_proj.VS.weight"].double()
    vu, vvs = sd[pre + "v_proj.U.weight"].double(), sd[pre + "v_proj.VS.weight"].double()
    c = 0
    for h, (r, o) in enumerate(zip(ranks, lw.k_head_offsets.tolist())):
        k_ref = x @ (ku[h * Hd:(h + 1) * Hd, c:c + r] @ kvs[c:c + r]).T
        k_got = codes[:, o:o + 16 * ((r + 15) // 16)] @ w.k_up[o:o + 16 * ((r + 15) // 16)].double()
        torch.testing.assert_close(k_got, k_ref, rtol=1e-5, atol=1e-5)
        c += r
    vc = codes[:, lw.k_width:]
    v_ref = (x @ (vu @ vvs).T).view(5, H, Hd)
    for hq in range(2 * H):
        torch.testing.assert_close(vc @ w.v_up_by_q[hq].double(), v_ref[:, hq // 2], rtol=1e-5, atol=1e-5)
