"""Context-parallel decode, host side, on two gloo ranks (CPU): each rank takes its
contiguous share of every sequence's 256-token tiles (the split the CUDA path
uses) and computes the partial (unnormalised lifted output, per-head max, softmax
denominator) of the reference decode math over those tokens. The partials are
exchanged with starkv_b200.context_parallel.gather_partials (one all-gather of
packed [out | m | l] buffers), and the combination the native combine kernel
applies (tested on the GPU), done here on the gathered data, must give the
unsplit decode of the oracle. Sequence lengths include ones with fewer tiles
than ranks (a rank with no token)."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2
LENS = [700, 31, 513, 256]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed=9, H=4):
    import starkv_oracle as O
    rng = np.random.default_rng(seed)
    ranks = [16, 32, 48, 16]
    _, offsets, W = O.k_layout(ranks)
    rv, Lmax = 64, max(LENS)
    seqs = []
    for L in LENS:
        k = rng.standard_normal((L, W))
        for r, o in zip(ranks, offsets):
            k[:, o + r:o + (-(-r // 16) * 16)] = 0.0
        seqs.append((rng.standard_normal((H, 128)), k, rng.standard_normal((L, rv))))
    k_up = rng.standard_normal((W, 128)) / 6
    v_up = rng.standard_normal((H, rv, 128)) / 8
    return ranks, offsets, seqs, k_up, v_up, O.rope_cos_sin(Lmax), 128 ** -0.5


def _partial(q, k_rows, v_rows, k_up, ranks, offsets, v_up, cs, scale, t0, t1):
    """Unnormalised lifted output, max and denominator over tokens [t0, t1)."""
    H = q.shape[0]
    out, m, l = np.zeros((H, 128)), np.full(H, -np.inf), np.zeros(H)
    if t1 <= t0:
        return out, m, l
    cos, sin = cs[t0:t1, :64], cs[t0:t1, 64:]
    for h in range(H):
        o, r = offsets[h], ranks[h]
        k = k_rows[t0:t1, o:o + r] @ k_up[o:o + r]
        kr = np.concatenate([k[:, :64] * cos - k[:, 64:] * sin, k[:, 64:] * cos + k[:, :64] * sin], 1)
        lg = kr @ q[h] * scale
        m[h] = lg.max()
        p = np.exp(lg - m[h])
        l[h] = p.sum()
        out[h] = (p @ v_rows[t0:t1]) @ v_up[h]
    return out, m, l


def _rank_main(rank, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        import starkv_oracle as O
        from starkv_b200.context_parallel import gather_partials
        ranks, offsets, seqs, k_up, v_up, cs, scale = _inputs()
        outs, ms, ls = [], [], []
        for (q, k, v), L in zip(seqs, LENS):
            T = -(-L // 256)
            s0, s1 = T * rank // WORLD, T * (rank + 1) // WORLD
            o, m, l = _partial(q, k, v, k_up, ranks, offsets, v_up, cs, scale, 256 * s0, min(256 * s1, L))
            outs.append(o); ms.append(m); ls.append(l)
        parts = gather_partials(torch.tensor(np.stack(outs)), torch.tensor(np.stack(ms)),
                                torch.tensor(np.stack(ls))).numpy()
        if rank == 0:
            # the combination starkv_cp_combine applies, on the gathered rank-major packed buffer
            n, H = len(LENS), ms[0].shape[0]
            P = parts.reshape(WORLD, -1)
            o = P[:, :n * H * 128].reshape(WORLD, n, H, 128)
            m = P[:, n * H * 128:n * H * 129].reshape(WORLD, n, H)
            l = P[:, n * H * 129:].reshape(WORLD, n, H)
            M = m.max(0)
            s = np.exp(m - M)
            got = (s[..., None] * o).sum(0) / (s * l).sum(0)[..., None]
            ref = np.stack([O.attend_one(q, k, v, k_up, ranks, offsets, 1, v_up, cs, scale) for q, k, v in seqs])
            result["err"] = float(np.abs(got - ref).max())
            result["scale"] = float(np.abs(ref).max())
    finally:
        dist.destroy_process_group()


def test_two_rank_context_split_matches_unsplit_decode():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
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
        assert result["err"] <= 1e-10 * max(1.0, result["scale"]), result["err"]


def _page_rank_main(rank, port, result):
    """Page round-robin placement (the whole model's split for growing sequences):
    the rank's pages of a sequence, as one local sequence, with the rank's permuted
    rotary table (context_parallel.local_rotary_table), give partials that combine
    to the unsplit decode."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        import starkv_oracle as O
        from starkv_b200 import context_parallel as cp
        ranks, offsets, seqs, k_up, v_up, cs, scale = _inputs()
        cs_local = cp.local_rotary_table(torch.tensor(cs), rank, WORLD).numpy()
        outs, ms, ls = [], [], []
        for (q, k, v), L in zip(seqs, LENS):
            pos = np.arange(L)
            mine = pos[cp.page_owner(pos, WORLD) == rank]
            assert np.array_equal(cp.local_index(mine, WORLD), np.arange(mine.size))
            n_loc = int(cp.local_len(L, rank, WORLD))
            assert n_loc == mine.size
            o, m, l = _partial(q, k[mine], v[mine], k_up, ranks, offsets, v_up, cs_local, scale, 0, n_loc)
            outs.append(o); ms.append(m); ls.append(l)
        parts = cp.gather_partials(torch.tensor(np.stack(outs)), torch.tensor(np.stack(ms)),
                                   torch.tensor(np.stack(ls))).numpy()
        if rank == 0:
            n, H = len(LENS), ms[0].shape[0]
            P = parts.reshape(WORLD, -1)
            o = P[:, :n * H * 128].reshape(WORLD, n, H, 128)
            m = P[:, n * H * 128:n * H * 129].reshape(WORLD, n, H)
            l = P[:, n * H * 129:].reshape(WORLD, n, H)
            M = m.max(0)
            s = np.exp(m - M)
            got = (s[..., None] * o).sum(0) / (s * l).sum(0)[..., None]
            ref = np.stack([O.attend_one(q, k, v, k_up, ranks, offsets, 1, v_up, cs, scale) for q, k, v in seqs])
            result["err"] = float(np.abs(got - ref).max())
            result["scale"] = float(np.abs(ref).max())
    finally:
        dist.destroy_process_group()


def test_two_rank_page_split_matches_unsplit_decode():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_page_rank_main, args=(r, port, result)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert result["scale"] > 0
        assert result["err"] <= 1e-10 * max(1.0, result["scale"]), result["err"]


def _agree_rank_main(rank, port, result):
    """Rank 1 has fewer cache blocks than rank 0: extend_agreed refuses on both
    ranks, neither table moves, and after a release both extend together."""
    from starkv_b200 import context_parallel as cp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        t = cp.PageSplitTables(rank, WORLD, 64 if rank == 0 else 3)
        cp.extend_agreed(t, "a", 48)
        cp.extend_agreed(t, "b", 40)
        before = (dict(t.lens), {k: list(v) for k, v in t.blocks.items()}, list(t.free))
        refused = False
        try:
            cp.extend_agreed(t, "a", 32)          # rank 1 is out of blocks
        except RuntimeError:
            refused = True
        same = before == (dict(t.lens), {k: list(v) for k, v in t.blocks.items()}, list(t.free))
        t.release("b")
        slots = cp.extend_agreed(t, "a", 32)
        result[rank] = (refused, same, t.lens["a"], sum(s >= 0 for s in slots))
    finally:
        dist.destroy_process_group()


def test_two_rank_page_split_extension_is_agreed_by_all_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_agree_rank_main, args=(r, port, result)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = dict(result)
    assert all(res[r][0] and res[r][1] for r in range(WORLD))      # both refused, nothing changed
    assert [res[r][2] for r in range(WORLD)] == [80, 80]             # both grew together afterwards
    assert res[0][3] + res[1][3] == 32                               # each new token on exactly one rank
