"""CPU checks of the attention layer's host logic (starkv_b200.layer) and the model
config: how a tensor-parallel shard slices the weights, and that folding the 3.2-bit
rotations into the factors leaves every head's K and V products unchanged."""
import pytest
import torch

from starkv_b200 import layer as Ly
from starkv_b200 import sharding
from starkv_b200.workload import sample_ranks

HIDDEN, HEADS = 256, 8


def weights(hkv=None, seed=2):
    ranks, rv = sample_ranks(hkv or HEADS, seed)
    return Ly.random_weights(HIDDEN, HEADS, ranks, rv, seed=seed, num_kv_heads=hkv, device="cpu",
                             dtype=torch.float32)


@pytest.mark.parametrize("world,hkv", [(2, None), (4, None), (2, 4)])
def test_shards_partition_heads_and_slice_weights(world, hkv):
    w = weights(hkv)
    cs = torch.randn(16, 128)
    shards = [Ly.StarKVAttentionLayer(w, cs, rank=r, world=world) for r in range(world)]
    kv_heads = sorted(h for s in shards for h in s.heads)
    assert kv_heads == list(range(w.num_kv_heads))
    q_heads = sorted(h for s in shards for h in s.q_heads)
    assert q_heads == list(range(w.num_heads))
    W_full = sum(sharding.align16(r) for r in w.k_ranks)
    for s in shards:
        qh = torch.tensor(s.q_heads)
        assert torch.equal(s.wq, w.wq.view(HEADS, 128, HIDDEN)[qh].reshape(-1, HIDDEN))
        assert torch.equal(s.wo, w.wo.view(HIDDEN, HEADS, 128)[:, qh].reshape(HIDDEN, -1))
        assert torch.equal(s.v_up_by_q, w.v_up_by_q[qh])
        _, _, _, lanes = sharding.shard_lanes(w.k_ranks, s.heads)
        assert torch.equal(s.kv_down[:s.k_width], w.kv_down[torch.tensor(lanes)])
        assert torch.equal(s.kv_down[s.k_width:], w.kv_down[W_full:])       # V replicated
        assert torch.equal(s.k_up, w.k_up[torch.tensor(lanes)])
    # the shards' output columns add up to the whole o_proj
    whole = Ly.StarKVAttentionLayer(w, cs)
    x = torch.randn(3, HEADS * 128)
    parts = sum(x.view(3, HEADS, 128)[:, torch.tensor(s.q_heads)].reshape(3, -1) @ s.wo.t() for s in shards)
    torch.testing.assert_close(parts, x @ whole.wo.t(), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("world", [1, 2])
def test_folded_rotations_keep_k_and_v_products(world):
    """3.2-bit layer: codes come out of kv_down rotated, and codes . k_up (per head)
    and v_codes . v_up_by_q equal the unrotated products."""
    w = weights()
    cs = torch.randn(16, 128)
    h = torch.randn(5, HIDDEN)
    for r in range(world):
        plain = Ly.StarKVAttentionLayer(w, cs, quant=False, rank=r, world=world)
        rot = Ly.StarKVAttentionLayer(w, cs, quant=True, rank=r, world=world)
        kp, vp = plain.codes(h)
        kr, vr = rot.codes(h)
        assert not torch.allclose(kp, kr)                      # the stored basis differs ...
        for rk, o in zip(plain.k_ranks_host, plain.k_head_offsets.tolist()):
            torch.testing.assert_close(kr[:, o:o + rk] @ rot.k_up[o:o + rk], kp[:, o:o + rk] @ plain.k_up[o:o + rk],
                                       rtol=1e-4, atol=1e-4)   # ... the lifted K does not
        torch.testing.assert_close(torch.einsum("tr,hrd->thd", vr, rot.v_up_by_q),
                                   torch.einsum("tr,hrd->thd", vp, plain.v_up_by_q), rtol=1e-4, atol=1e-4)


def test_shard_rotations_match_whole_layer():
    """A shard uses the same per-head rotations as the whole layer, so its codes
    equal the whole layer's codes of its heads."""
    w = weights()
    cs = torch.randn(16, 128)
    h = torch.randn(4, HIDDEN)
    whole = Ly.StarKVAttentionLayer(w, cs, quant=True)
    kw, vw = whole.codes(h)
    for r in range(2):
        s = Ly.StarKVAttentionLayer(w, cs, quant=True, rank=r, world=2)
        ks, vs = s.codes(h)
        _, _, _, lanes = sharding.shard_lanes(w.k_ranks, s.heads)
        torch.testing.assert_close(ks, kw[:, torch.tensor(lanes)], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(vs, vw, rtol=1e-5, atol=1e-5)


def test_model_config_rank_sampler():
    from starkv_b200.model import ModelConfig
    cfg = ModelConfig()
    Ws, rvs = [], []
    for i in range(32):
        ranks, rv = cfg.layer_ranks(i)
        assert len(ranks) == 32 and all(r in (16, 32, 48) for r in ranks) and rv % 32 == 0
        Ws.append(sum(sharding.align16(r) for r in ranks))
        rvs.append(rv)
    assert 850 < sum(Ws) / 32 < 1150 and 1100 < sum(rvs) / 32 < 1450    # comp-ratio 0.75 sizes
    assert cfg.layer_ranks(5) == ModelConfig().layer_ranks(5)           # seeded: every rank agrees


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_page_round_robin_placement(world):
    """Every global position has one owner and a distinct local index there, the local
    tokens of a rank are a contiguous prefix of length local_len, global_position
    inverts local_index, and the rank's rotary table row i is the global row of its
    local token i."""
    from starkv_b200 import context_parallel as cp
    for L in [0, 1, 15, 16, 17, 47, 48, 200, 1029]:
        pos = torch.arange(L)
        owner = cp.page_owner(pos, world)
        for r in range(world):
            mine = pos[owner == r]
            li = cp.local_index(mine, world)
            assert torch.equal(li, torch.arange(mine.numel()))                  # contiguous local prefix
            assert int(cp.local_len(L, r, world)) == mine.numel()
            assert torch.equal(cp.global_position(li, r, world), mine)
        lens = torch.tensor([L, L + 1])
        assert torch.equal(cp.local_len(lens, 0, world),
                           torch.tensor([int(cp.local_len(L, 0, world)), int(cp.local_len(L + 1, 0, world))]))
    cs = torch.randn(100, 128)
    for r in range(world):
        t = cp.local_rotary_table(cs, r, world)
        i = torch.arange(t.shape[0])
        g = cp.global_position(i, r, world)
        ok = g < 100
        assert torch.equal(t[ok], cs[g[ok]])
        assert t.shape[0] * world >= 100


def test_model_rejects_unknown_attention_split():
    from starkv_b200.model import ModelConfig, StarKVModel
    with pytest.raises(ValueError):
        StarKVModel(ModelConfig(layers=1), "cpu", attn_parallel="rows")


@pytest.mark.parametrize("world", [1, 2, 4])
def test_page_split_tables_place_growing_sequences(world):
    """Sequences grow by prompts and single decode tokens while others finish. Every
    token is written on exactly one rank, at a slot that no other live token holds.
    Reading a rank's cache through its decode block table gives the rank's tokens in
    local order, with global positions global_position(i). Freed blocks are reused,
    and a rank with too few blocks refuses without changing its state."""
    import random
    import numpy as np
    from starkv_b200 import context_parallel as cp
    rng = random.Random(world)
    nb = 2 + 16 // world                 # small enough that ranks run short during the walk
    tabs = [cp.PageSplitTables(r, world, nb) for r in range(world)]
    refused = 0
    caches = [np.full((nb, 16), -1, dtype=np.int64) for _ in range(world)]   # global position stored per slot
    live, next_id = {}, 0
    for step in range(300):
        if len(live) < 4 and rng.random() < 0.3:
            sid, n = next_id, rng.randint(1, 60)
            next_id += 1
            live[sid] = 0
        elif live and rng.random() < 0.05:
            sid = rng.choice(list(live))
            for t in tabs:
                t.release(sid)
            del live[sid]
            continue
        elif live:
            sid, n = rng.choice(list(live)), 1
        else:
            continue
        try:
            slots = cp.extend_on_all_ranks(tabs, sid, n)
        except RuntimeError:
            refused += 1
            assert all(t.lens.get(sid, 0) == live[sid] for t in tabs)   # no rank moved
            continue                      # a rank is short: no rank extended
        L0 = live[sid]
        for i in range(n):
            owners = [r for r in range(world) if slots[r][i] >= 0]
            assert owners == [int(cp.page_owner(L0 + i, world))]
            r = owners[0]
            caches[r].reshape(-1)[slots[r][i]] = L0 + i
        live[sid] = L0 + n
        # every live sequence reads back in local order on every rank
        for r, t in enumerate(tabs):
            ids = list(live)
            bt, lens, mx = t.decode_metadata(ids)
            for k, s in enumerate(ids):
                ln = int(lens[k])
                assert ln == int(cp.local_len(live[s], r, world))
                idx = np.arange(ln)
                got = caches[r][bt[k, idx // 16].numpy(), idx % 16]
                assert np.array_equal(got, cp.global_position(idx, r, world)), (step, r, s)
            assert mx >= max([int(x) for x in lens] + [1])
            held = [b for s in ids for b in t.blocks.get(s, [])]
            assert len(held) == len(set(held)) and 0 not in held      # no block twice, null block kept
            assert len(held) + len(t.free) == nb - 1                  # freed blocks go back to the pool
    assert refused > 0                    # the refusal path ran
    # a refused extension leaves the tables as they were
    t = cp.PageSplitTables(0, world, 3)
    t.extend("a", 16)
    before = (dict(t.lens), {k: list(v) for k, v in t.blocks.items()}, list(t.free))
    with pytest.raises(RuntimeError):
        t.extend("a", 16 * world * 4)
    assert before == (dict(t.lens), {k: list(v) for k, v in t.blocks.items()}, list(t.free))


def test_page_split_refusal_keeps_all_ranks_consistent():
    """Rank 1 is short of blocks while rank 0 is not: the group refuses as a whole,
    every rank keeps its lengths and its pool intact, and the sequence can still grow
    once rank 1 frees blocks."""
    from starkv_b200 import context_parallel as cp
    tabs = [cp.PageSplitTables(0, 2, 64), cp.PageSplitTables(1, 2, 3)]   # rank 1: 2 usable blocks
    cp.extend_on_all_ranks(tabs, "a", 48)            # pages 0, 2 on rank 0; page 1 on rank 1
    cp.extend_on_all_ranks(tabs, "b", 40)            # rank 1 takes its second (last) block
    assert not tabs[1].free and tabs[1].blocks_needed("a", 32) == 1
    assert tabs[0].can_extend("a", 32) and not tabs[1].can_extend("a", 32)
    before = [(dict(t.lens), {k: list(v) for k, v in t.blocks.items()}, list(t.free)) for t in tabs]
    with pytest.raises(RuntimeError):
        cp.extend_on_all_ranks(tabs, "a", 32)
    assert before == [(dict(t.lens), {k: list(v) for k, v in t.blocks.items()}, list(t.free)) for t in tabs]
    for t in tabs:
        t.release("b")
    slots = cp.extend_on_all_ranks(tabs, "a", 32)
    assert [t.lens["a"] for t in tabs] == [80, 80]
    assert sum(s >= 0 for s in slots[0]) + sum(s >= 0 for s in slots[1]) == 32
