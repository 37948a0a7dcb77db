"""GPU parity of one compressed attention layer's decode step (starkv_b200.layer):
Q projection + rotary, K/V down-projection to codes, cache write (bf16) or pack
(3.2-bit), paged decode, o_proj - and its head-sharded tensor-parallel split.

The reference recomputes the attention with the CPU oracle (fp64) from exactly the
cache rows and rotated queries the GPU produced, then applies o_proj in fp64.
Tolerance (the target's): 2e-2 abs + 1e-2 rel.
"""
import numpy as np
import pytest
import torch

import starkv_oracle as O

pytestmark = pytest.mark.gpu

LENS = [1, 40, 300, 1029]
HIDDEN, HEADS = 512, 8


def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def setup(quant, world=1, seed=3):
    """Weights, one layer per rank, and for each rank a cache holding the codes of
    every sequence's past tokens (positions 0 .. L-2) computed from seeded hidden
    states; returns (layers, caches, block_table, seq_lens, hidden_new, positions, slots)."""
    from starkv_b200 import layer as Ly
    from starkv_b200.workload import rope_cos_sin, sample_ranks
    dev = cuda()
    ranks, rv = sample_ranks(HEADS, seed)
    w = Ly.random_weights(HIDDEN, HEADS, ranks, rv, seed=seed, device=dev)
    cs = rope_cos_sin(2048, dev)
    layers = [Ly.StarKVAttentionLayer(w, cs, quant=quant, rank=r, world=world) for r in range(world)]
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    npages = [-(-L // 16) for L in LENS]
    perm = torch.randperm(sum(npages), generator=torch.Generator().manual_seed(seed)) + 1
    bt = torch.zeros(len(LENS), max(npages), dtype=torch.int32)
    k = 0
    for b, p in enumerate(npages):
        bt[b, :p] = perm[k:k + p]
        k += p
    bt = bt.to(dev)
    caches = []
    hist = [torch.randn(L, HIDDEN, generator=g, device=dev).to(torch.bfloat16) for L in LENS]
    for ly in layers:
        width, dt = ly.cache_row()
        cache = torch.zeros(sum(npages) + 1, 16, width, dtype=dt, device=dev)
        for b, L in enumerate(LENS):
            if L > 1:
                pos = torch.arange(L - 1, device=dev)
                slots = bt[b, pos // 16].long() * 16 + pos % 16
                kc, vc = ly.codes(hist[b][:L - 1])
                if quant:
                    from starkv_b200.kernels import paged_quant as pq
                    pq.pack_kv(kc, vc, cache, slots, ly.row, ly.k_ranks, ly.k_head_offsets, ly.k_nouts)
                else:
                    from starkv_b200.kernels.paged_decode import write_kv_bf16
                    write_kv_bf16(kc, vc, cache, slots)
        caches.append(cache)
    new = torch.stack([h[-1] for h in hist])
    positions = torch.tensor([L - 1 for L in LENS], device=dev)
    slots = bt[torch.arange(len(LENS), device=dev), positions // 16].long() * 16 + positions % 16
    seq_lens = torch.tensor(LENS, dtype=torch.int32, device=dev)
    return layers, caches, bt, seq_lens, new, positions, slots


def reference(ly, cache, bt, new, positions):
    """fp64 oracle attention over the stored cache rows + o_proj."""
    from starkv_b200.layer import rope
    f = lambda t: t.double().cpu().numpy()  # noqa: E731
    q = rope(torch.nn.functional.linear(new, ly.wq).view(len(LENS), ly.num_heads, 128), positions,
             ly.cos_sin_cache)
    outs = []
    row = O.QuantRow(ly.k_width, ly.num_kv_heads, ly.v_rank) if ly.quant else None
    offs = ly.k_head_offsets.tolist()
    for b, L in enumerate(LENS):
        pos = torch.arange(L, device=cache.device)
        rows = cache[bt[b, pos // 16].long(), pos % 16].cpu()
        if ly.quant:
            kd, vd = O.unpack_rows(rows.numpy(), row, ly.k_ranks_host)
        else:
            r = rows.double().numpy()
            kd, vd = r[:, :ly.k_width], r[:, ly.k_width:]
        outs.append(O.attend_one(f(q[b]), kd, vd, f(ly.k_up), ly.k_ranks_host, offs,
                                 ly.num_heads // ly.num_kv_heads, f(ly.v_up_by_q), f(ly.cos_sin_cache), ly.scale))
    attn = np.stack(outs).reshape(len(LENS), -1)
    return attn @ f(ly.wo).T


@pytest.mark.parametrize("quant", [False, True])
def test_layer_decode_step_vs_oracle(quant):
    layers, caches, bt, seq_lens, new, positions, slots = setup(quant)
    ly, cache = layers[0], caches[0]
    out = ly.forward(new, positions, cache, bt, seq_lens, max(LENS), slots)
    assert out.shape == (len(LENS), HIDDEN) and out.dtype == torch.bfloat16
    # the step's own codes landed in the cache at their slots
    kc, vc = ly.codes(new)
    got_rows = cache.view(-1, cache.shape[-1])[slots]
    if quant:
        ref_rows = O.pack_rows(kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                               O.QuantRow(ly.k_width, ly.num_kv_heads, ly.v_rank), ly.k_ranks_host)
        np.testing.assert_array_equal(got_rows.cpu().numpy(), ref_rows)
    else:
        assert torch.equal(got_rows, torch.cat([kc, vc], dim=-1))
    ref = reference(ly, cache, bt, new, positions)
    got = out.double().cpu().numpy()
    err = np.abs(got - ref)
    assert np.all(err <= 2e-2 + 1e-2 * np.abs(ref)), f"max abs err {err.max():.3e}"


@pytest.mark.parametrize("quant", [False, True])
def test_layer_decode_step_with_padding_rows(quant):
    """A CUDA-graph padded batch (attention.py:181, 199): two padding rows with slot
    -1, length 0 and an all-zero block table row ride along with the real rows. They
    write their codes to the reserved null block (slot -1 -> block 0, position 0),
    attend to that one position (length clamped to 1) and give a finite output equal
    to the oracle's over the row that landed there; the real rows are unchanged."""
    from starkv_b200.layer import rope
    layers, caches, bt, seq_lens, new, positions, slots = setup(quant)
    ly, cache = layers[0], caches[0]
    dev, n, P = new.device, len(LENS), 2
    g = torch.Generator(device=dev).manual_seed(99)
    pad_hidden = torch.randn(P, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    out = ly.forward(torch.cat([new, pad_hidden]), torch.cat([positions, torch.zeros(P, dtype=positions.dtype,
                                                                                     device=dev)]),
                     cache, torch.cat([bt, torch.zeros(P, bt.shape[1], dtype=bt.dtype, device=dev)]),
                     torch.cat([seq_lens, torch.zeros(P, dtype=seq_lens.dtype, device=dev)]), max(LENS),
                     torch.cat([slots, torch.full((P,), -1, dtype=slots.dtype, device=dev)]))
    got = out.double().cpu().numpy()
    assert np.isfinite(got).all()
    ref = reference(ly, cache, bt, new, positions)
    assert np.all(np.abs(got[:n] - ref) <= 2e-2 + 1e-2 * np.abs(ref))
    # padding rows: the oracle over the single null-block position 0, whatever row landed there
    f = lambda t: t.double().cpu().numpy()  # noqa: E731
    rows = cache[0, :1].cpu()
    if quant:
        kd, vd = O.unpack_rows(rows.numpy(), O.QuantRow(ly.k_width, ly.num_kv_heads, ly.v_rank), ly.k_ranks_host)
    else:
        r = rows.double().numpy()
        kd, vd = r[:, :ly.k_width], r[:, ly.k_width:]
    qp = rope(torch.nn.functional.linear(pad_hidden, ly.wq).view(P, ly.num_heads, 128),
              torch.zeros(P, dtype=torch.long, device=dev), ly.cos_sin_cache)
    for i in range(P):
        a = O.attend_one(f(qp[i]), kd, vd, f(ly.k_up), ly.k_ranks_host, ly.k_head_offsets.tolist(),
                         ly.num_heads // ly.num_kv_heads, f(ly.v_up_by_q), f(ly.cos_sin_cache), ly.scale)
        refp = a.reshape(-1) @ f(ly.wo).T
        assert np.all(np.abs(got[n + i] - refp) <= 2e-2 + 1e-2 * np.abs(refp))


@pytest.mark.parametrize("quant", [False, True])
def test_layer_head_shards_sum_to_whole(quant):
    """Two head shards (LPT) on one GPU: their o_proj partial sums add up to the
    whole layer's output (the all-reduce of a 2-rank group)."""
    whole, wc, bt, seq_lens, new, positions, slots = setup(quant, world=1)
    shards, sc, *_ = setup(quant, world=2)
    full = whole[0].forward(new, positions, wc[0], bt, seq_lens, max(LENS), slots).float()
    parts = [ly.forward(new, positions, c, bt, seq_lens, max(LENS), slots, reduce=False).float()
             for ly, c in zip(shards, sc)]
    assert sorted(shards[0].heads + shards[1].heads) == list(range(HEADS))
    got = (parts[0] + parts[1]).cpu().numpy()
    ref = full.cpu().numpy()
    err = np.abs(got - ref)
    assert np.all(err <= 2e-2 + 2e-2 * np.abs(ref)), f"max abs err {err.max():.3e}"


PROMPTS = [5, 23, 64]


def prefill_setup(quant, world=1, seed=11, num_kv_heads=None):
    from starkv_b200 import layer as Ly
    from starkv_b200.workload import rope_cos_sin, sample_ranks
    dev = cuda()
    hkv = num_kv_heads or HEADS
    ranks, rv = sample_ranks(hkv, seed)
    w = Ly.random_weights(HIDDEN, HEADS, ranks, rv, seed=seed, num_kv_heads=hkv, device=dev)
    cs = rope_cos_sin(256, dev)
    layers = [Ly.StarKVAttentionLayer(w, cs, quant=quant, rank=r, world=world) for r in range(world)]
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    T = sum(PROMPTS)
    hidden = torch.randn(T, HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    positions = torch.cat([torch.arange(L, device=dev) for L in PROMPTS])
    slots = torch.randperm(T + 16, generator=torch.Generator().manual_seed(seed))[:T].to(dev) + 16
    caches = []
    for ly in layers:
        width, dt = ly.cache_row()
        caches.append(torch.zeros(-(-(T + 32) // 16), 16, width, dtype=dt, device=dev))
    return layers, caches, hidden, positions, slots


def prefill_reference(ly, hidden, positions):
    """fp64 oracle: each prompt token attends causally over the prompt's own (not
    quantized) codes, then o_proj."""
    from starkv_b200.layer import rope
    f = lambda t: t.double().cpu().numpy()  # noqa: E731
    T = hidden.shape[0]
    q = rope(torch.nn.functional.linear(hidden, ly.wq).view(T, ly.num_heads, 128), positions, ly.cos_sin_cache)
    kc, vc = ly.codes(hidden)
    kc, vc, qn = f(kc), f(vc), f(q)
    offs = ly.k_head_offsets.tolist()
    outs, s0 = [], 0
    for L in PROMPTS:
        for t in range(L):
            outs.append(O.attend_one(qn[s0 + t], kc[s0:s0 + t + 1], vc[s0:s0 + t + 1], f(ly.k_up), ly.k_ranks_host,
                                     offs, ly.num_heads // ly.num_kv_heads, f(ly.v_up_by_q), f(ly.cos_sin_cache),
                                     ly.scale))
        s0 += L
    return np.stack(outs).reshape(T, -1) @ f(ly.wo).T


@pytest.mark.parametrize("quant,hkv", [(False, None), (False, 4), (True, None)])
def test_layer_prefill_vs_oracle(quant, hkv):
    layers, caches, hidden, positions, slots = prefill_setup(quant, num_kv_heads=hkv)
    ly, cache = layers[0], caches[0]
    out = ly.prefill(hidden, positions, PROMPTS, cache, slots)
    assert out.shape == (hidden.shape[0], HIDDEN)
    kc, vc = ly.codes(hidden)
    got_rows = cache.view(-1, cache.shape[-1])[slots.long()]
    if quant:
        ref_rows = O.pack_rows(kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                               O.QuantRow(ly.k_width, ly.num_kv_heads, ly.v_rank), ly.k_ranks_host)
        np.testing.assert_array_equal(got_rows.cpu().numpy(), ref_rows)
    else:
        assert torch.equal(got_rows, torch.cat([kc, vc], dim=-1))
    ref = prefill_reference(ly, hidden, positions)
    err = np.abs(out.double().cpu().numpy() - ref)
    assert np.all(err <= 2e-2 + 1e-2 * np.abs(ref)), f"max abs err {err.max():.3e}"


def test_layer_prefill_head_shards_sum_to_whole():
    whole, wc, hidden, positions, slots = prefill_setup(False)
    shards, sc, *_ = prefill_setup(False, world=2)
    full = whole[0].prefill(hidden, positions, PROMPTS, wc[0], slots).float()
    parts = [ly.prefill(hidden, positions, PROMPTS, c, slots, reduce=False).float() for ly, c in zip(shards, sc)]
    err = ((parts[0] + parts[1]) - full).abs()
    assert bool((err <= 2e-2 + 2e-2 * full.abs()).all()), f"max abs err {err.max().item():.3e}"
