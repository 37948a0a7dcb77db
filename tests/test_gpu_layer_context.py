"""GPU parity of the page-split (context-parallel) attention layer
(starkv_b200.layer.StarKVContextLayer), its ranks emulated in one process: each rank
holds page p % world of every sequence as its own local sequence, writes the new
token where it owns the page, decodes all heads over its pages with its permuted
rotary table, and the partials are combined (context_parallel.combine_local, the
same native combine the all-gather path uses) and go through o_proj.

Reference: the fp64 CPU oracle over the whole layer's cache (the same codes at
global positions), and the whole layer's own GPU step. Tolerance (the target's):
2e-2 abs + 1e-2 rel.
"""
import numpy as np
import pytest
import torch

from test_gpu_layer import HEADS, HIDDEN, LENS, cuda, reference, setup

pytestmark = pytest.mark.gpu


def local_setup(w, cs, quant, rank, world, whole_cache, bt, seed=3):
    """One rank's layer, local cache (rows of positions 0 .. L-2 that it owns, copied
    from the whole layer's cache), local block table, seq_lens and the new token's slot."""
    from starkv_b200 import context_parallel as cp
    from starkv_b200.layer import StarKVContextLayer
    dev = whole_cache.device
    ly = StarKVContextLayer(w, cs, quant=quant, rank=rank, world=world)
    llen = [int(cp.local_len(L, rank, world)) for L in LENS]
    lpages = [-(-x // 16) for x in llen]
    tot = max(sum(lpages), 1)
    perm = torch.randperm(tot, generator=torch.Generator().manual_seed(seed + 10 * rank)) + 1
    lbt = torch.zeros(len(LENS), max(max(lpages), 1), dtype=torch.int32)
    k = 0
    for b, p in enumerate(lpages):
        lbt[b, :p] = perm[k:k + p]
        k += p
    lbt = lbt.to(dev)
    cache = torch.zeros(tot + 1, 16, whole_cache.shape[-1], dtype=whole_cache.dtype, device=dev)
    for b, L in enumerate(LENS):
        pos = torch.arange(L - 1, device=dev)
        mine = pos[cp.page_owner(pos, world) == rank]
        if mine.numel():
            li = cp.local_index(mine, world)
            cache[lbt[b, li // 16].long(), li % 16] = whole_cache[bt[b, mine // 16].long(), mine % 16]
    newpos = torch.tensor([L - 1 for L in LENS], device=dev)
    li = cp.local_index(newpos, world)
    slots = lbt[torch.arange(len(LENS), device=dev), (li // 16).clamp(max=lbt.shape[1] - 1)].long() * 16 + li % 16
    slots = torch.where(cp.page_owner(newpos, world) == rank, slots, torch.full_like(slots, -1))
    seq_lens = torch.tensor(llen, dtype=torch.int32, device=dev)
    return ly, cache, lbt, seq_lens, max(max(llen), 1), slots


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("quant", [False, True])
def test_page_split_layer_equals_whole_layer(quant, world):
    from starkv_b200 import context_parallel as cp
    from starkv_b200 import layer as Ly
    from starkv_b200.workload import rope_cos_sin, sample_ranks
    dev = cuda()
    layers, caches, bt, seq_lens, new, positions, slots = setup(quant)
    whole, wcache = layers[0], caches[0]
    ranks, rv = sample_ranks(HEADS, 3)
    w = Ly.random_weights(HIDDEN, HEADS, ranks, rv, seed=3, device=dev)   # the same weights as setup()'s
    cs = rope_cos_sin(2048, dev)
    parts, ranks_state = [], []
    for r in range(world):
        ly, cache, lbt, lsl, lmax, lslots = local_setup(w, cs, quant, r, world, wcache, bt)
        parts.append(ly.forward_partial(new, positions, cache, lbt, lsl, lmax, lslots))
        ranks_state.append((ly, cache, lbt, lslots))
    attn = cp.combine_local(parts, dtype=torch.bfloat16)
    got = torch.nn.functional.linear(attn.reshape(len(LENS), -1), ranks_state[0][0].wo)
    # the new token's codes went to its owner's local slot only
    kc, vc = whole.codes(new)
    for b, L in enumerate(LENS):
        owner = int(cp.page_owner(L - 1, world))
        for r, (ly, cache, lbt, lslots) in enumerate(ranks_state):
            assert (int(lslots[b]) >= 0) == (r == owner)
        ly, cache, lbt, lslots = ranks_state[owner]
        row = cache.view(-1, cache.shape[-1])[lslots[b]]
        if not quant:
            assert torch.equal(row, torch.cat([kc[b], vc[b]]))
    ref_out = whole.forward(new, positions, wcache, bt, seq_lens, max(LENS), slots)
    ref = reference(whole, wcache, bt, new, positions)
    g = got.double().cpu().numpy()
    err = np.abs(g - ref)
    assert np.all(err <= 2e-2 + 1e-2 * np.abs(ref)), f"vs oracle: max abs err {err.max():.3e}"
    w_err = np.abs(g - ref_out.double().cpu().numpy())
    assert np.all(w_err <= 2e-2 + 1e-2 * np.abs(ref)), f"vs whole layer: max abs err {w_err.max():.3e}"


@pytest.mark.parametrize("quant", [False, True])
def test_page_split_prefill_then_decode(quant):
    """Prompts prefilled through each rank's StarKVContextLayer (the inherited dense
    prefill, given the rank's local slots and -1 elsewhere), then one decode step:
    every rank's cache rows equal the whole layer's rows at the positions it owns,
    the prefill output equals the whole layer's, and the decode matches it."""
    from starkv_b200 import context_parallel as cp
    from starkv_b200 import layer as Ly
    from starkv_b200.workload import rope_cos_sin, sample_ranks
    dev = cuda()
    world, P = 2, [37, 70, 16]
    ranks, rv = sample_ranks(HEADS, 5)
    w = Ly.random_weights(HIDDEN, HEADS, ranks, rv, seed=5, device=dev)
    cs = rope_cos_sin(1024, dev)
    g = torch.Generator(device=dev).manual_seed(6)
    prompt = torch.randn(sum(P), HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    new = torch.randn(len(P), HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    ppos = torch.cat([torch.arange(L, device=dev) for L in P])
    seq_of = torch.cat([torch.full((L,), b, device=dev) for b, L in enumerate(P)])
    npos = torch.tensor(P, device=dev)                        # the decode token of each sequence

    whole = Ly.StarKVAttentionLayer(w, cs, quant=quant)
    pages = [-(-(L + 1) // 16) for L in P]
    bt = torch.zeros(len(P), max(pages), dtype=torch.int32)
    k = 1
    for b, p in enumerate(pages):
        bt[b, :p] = torch.arange(k, k + p)
        k += p
    bt = bt.to(dev)
    width, dt = whole.cache_row()
    wcache = torch.zeros(k, 16, width, dtype=dt, device=dev)
    pre_whole = whole.prefill(prompt, ppos, P, wcache, bt[seq_of, ppos // 16].long() * 16 + ppos % 16)
    dec_whole = whole.forward(new, npos, wcache, bt, torch.tensor([L + 1 for L in P], dtype=torch.int32, device=dev),
                              max(P) + 1, bt[torch.arange(len(P), device=dev), npos // 16].long() * 16 + npos % 16)

    parts = []
    for r in range(world):
        ly = Ly.StarKVContextLayer(w, cs, quant=quant, rank=r, world=world)
        llen = [int(cp.local_len(L + 1, r, world)) for L in P]
        lpages = [max(-(-x // 16), 1) for x in llen]
        lbt = torch.zeros(len(P), max(lpages), dtype=torch.int32)
        k = 1
        for b, p in enumerate(lpages):
            lbt[b, :p] = torch.arange(k, k + p)
            k += p
        lbt = lbt.to(dev)
        cache = torch.zeros(k, 16, width, dtype=dt, device=dev)

        def local_slots(seq, pos):
            li = cp.local_index(pos, world)
            s = lbt[seq, (li // 16).clamp(max=lbt.shape[1] - 1)].long() * 16 + li % 16
            return torch.where(cp.page_owner(pos, world) == r, s, torch.full_like(s, -1))

        pre = ly.prefill(prompt, ppos, P, cache, local_slots(seq_of, ppos))
        torch.testing.assert_close(pre, pre_whole, rtol=1e-2, atol=1e-3)   # the same math on the same inputs
        seqs = torch.arange(len(P), device=dev)
        parts.append(ly.forward_partial(new, npos, cache, lbt, torch.tensor(llen, dtype=torch.int32, device=dev),
                                        max(max(llen), 1), local_slots(seqs, npos)))
        # the rank's rows (prompt and decode token) are the whole layer's rows at its positions
        for b, L in enumerate(P):
            pos = torch.arange(L + 1, device=dev)
            mine = pos[cp.page_owner(pos, world) == r]
            li = cp.local_index(mine, world)
            got = cache[lbt[b, li // 16].long(), li % 16]
            ref = wcache[bt[b, mine // 16].long(), mine % 16]
            assert torch.equal(got, ref), (r, b)
        last_ly = ly
    attn = cp.combine_local(parts, dtype=torch.bfloat16)
    got = torch.nn.functional.linear(attn.reshape(len(P), -1), last_ly.wo).double()
    ref = dec_whole.double()
    err = (got - ref).abs()
    assert bool((err <= 2e-2 + 1e-2 * ref.abs()).all()), f"max abs err {float(err.max()):.3e}"


@pytest.mark.parametrize("quant", [False, True])
def test_page_split_tables_drive_prefill_and_growing_decode(quant):
    """Two emulated ranks, each with a context_parallel.PageSplitTables, prefill three
    prompts and then decode 24 steps. The steps cross page boundaries, so ownership of
    the new token alternates between the ranks. The 5-token prompt fits in page 0, so
    rank 1 starts with no token of that sequence (an empty block-table row, length 0,
    a partial with max -inf) and takes its first page at position 16 during the
    decode. Every step's combined output matches the whole layer's step."""
    from starkv_b200 import context_parallel as cp
    from starkv_b200 import layer as Ly
    from starkv_b200.workload import rope_cos_sin, sample_ranks
    dev = cuda()
    world, P, steps = 2, [5, 20, 45], 24
    ranks, rv = sample_ranks(HEADS, 7)
    w = Ly.random_weights(HIDDEN, HEADS, ranks, rv, seed=7, device=dev)
    cs = rope_cos_sin(1024, dev)
    g = torch.Generator(device=dev).manual_seed(8)
    prompt = torch.randn(sum(P), HIDDEN, generator=g, device=dev).to(torch.bfloat16)
    ppos = torch.cat([torch.arange(L, device=dev) for L in P])
    whole = Ly.StarKVAttentionLayer(w, cs, quant=quant)
    width, dt = whole.cache_row()
    wtab = cp.PageSplitTables(0, 1, 64)                 # world 1: the whole layer's own tables
    wcache = torch.zeros(64, 16, width, dtype=dt, device=dev)
    lys = [Ly.StarKVContextLayer(w, cs, quant=quant, rank=r, world=world) for r in range(world)]
    tabs = [cp.PageSplitTables(r, world, 64) for r in range(world)]
    caches = [torch.zeros(64, 16, width, dtype=dt, device=dev) for _ in range(world)]

    def slots_of(tab, counts):
        return torch.tensor([s for b, c in enumerate(counts) for s in tab.extend(b, c)], device=dev)

    whole.prefill(prompt, ppos, P, wcache, slots_of(wtab, P))
    for ly, tab, cache in zip(lys, tabs, caches):
        ly.prefill(prompt, ppos, P, cache, slots_of(tab, P))
    lens = list(P)
    assert tabs[1].local_len(0) == 0                    # rank 1 holds nothing of the short prompt yet
    for step in range(steps):
        new = torch.randn(len(P), HIDDEN, generator=g, device=dev).to(torch.bfloat16)
        pos = torch.tensor(lens, device=dev)
        ws = slots_of(wtab, [1] * len(P))
        bt, sl, mx = wtab.decode_metadata(range(len(P)), dev)
        ref = whole.forward(new, pos, wcache, bt, sl, mx, ws).double()
        parts = []
        for ly, tab, cache in zip(lys, tabs, caches):
            ls = slots_of(tab, [1] * len(P))
            lbt, lsl, lmx = tab.decode_metadata(range(len(P)), dev)
            parts.append(ly.forward_partial(new, pos, cache, lbt, lsl, lmx, ls))
        attn = cp.combine_local(parts, dtype=torch.bfloat16)
        got = torch.nn.functional.linear(attn.reshape(len(P), -1), lys[0].wo).double()
        err = (got - ref).abs()
        assert bool((err <= 2e-2 + 1e-2 * ref.abs()).all()), f"step {step}: max abs err {float(err.max()):.3e}"
        lens = [L + 1 for L in lens]
    assert tabs[1].local_len(0) == lens[0] - 16         # ...and took its first page during the decode
