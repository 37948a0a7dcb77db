"""Head-sharded decode on two ranks (gloo, CPU): each rank keeps the K codes,
k_up rows and query / v_up_by_q rows of its own KV heads and the whole V latent
(the host logic of starkv_b200.sharding), runs the reference decode math on its
shard, and the outputs gathered over the process group must equal the
unsharded decode. Attention needs no collective; the all-gather only collects
the result for the check."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(seed=5, n=3, Hkv=8, group=2, L=40):
    import starkv_oracle as O
    rng = np.random.default_rng(seed)
    ranks = [int(x) for x in rng.choice([16, 32, 48, 64], Hkv)]
    _, offsets, W = O.k_layout(ranks)
    rv = 96
    Hq = Hkv * group
    q = rng.standard_normal((n, Hq, 128))
    k_rows = rng.standard_normal((n, L, W))
    for r, o in zip(ranks, offsets):
        k_rows[:, :, o + r:o + (-(-r // 16) * 16)] = 0.0
    v_rows = rng.standard_normal((n, L, rv))
    k_up = rng.standard_normal((W, 128)) / 8
    v_up = rng.standard_normal((Hq, rv, 128)) / 10
    cs = O.rope_cos_sin(L)
    return dict(ranks=ranks, offsets=offsets, group=group, q=q, k_rows=k_rows, v_rows=v_rows, k_up=k_up,
                v_up=v_up, cs=cs, scale=128 ** -0.5)


def _decode(d, ranks, offsets, k_rows, k_up, q, v_up):
    import starkv_oracle as O
    return np.stack([O.attend_one(q[b], k_rows[b], d["v_rows"][b], k_up, ranks, offsets, d["group"], v_up,
                                  d["cs"], d["scale"]) for b in range(q.shape[0])])


def _rank_main(rank, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from starkv_b200.sharding import lpt_shard, query_heads, shard_lanes
        d = _layer()
        groups = lpt_shard(d["ranks"], WORLD)
        heads = groups[rank]
        lr, lo, _, lanes = shard_lanes(d["ranks"], heads)
        qh = query_heads(heads, d["group"])
        mine = _decode(d, lr, lo, d["k_rows"][:, :, lanes], d["k_up"][lanes], d["q"][:, qh], d["v_up"][qh])
        parts = [torch.zeros(mine.shape, dtype=torch.float64) for _ in range(WORLD)]
        dist.all_gather(parts, torch.from_numpy(mine))
        if rank == 0:
            full = _decode(d, d["ranks"], d["offsets"], d["k_rows"], d["k_up"], d["q"], d["v_up"])
            got = np.zeros_like(full)
            for r, g in enumerate(groups):
                got[:, query_heads(g, d["group"])] = parts[r].numpy()
            result["err"] = float(np.abs(got - full).max())
            result["scale"] = float(np.abs(full).max())
    finally:
        dist.destroy_process_group()


def test_two_rank_head_sharding_matches_unsharded_decode():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        result = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, port, result)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert result["scale"] > 0
        assert result["err"] <= 1e-12 * max(1.0, result["scale"])
