"""Benchmark of the STAR-KV paged low-rank decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode step of one compressed layer over the whole batch: write
the step's new K/V codes into the paged cache, then paged low-rank decode
attention (bf16 codes: configuration 2 of BASELINE.json, 64 sequences x 8192
tokens). The 3.2-bit configuration 3 (64 x 16384) is measured the same way and
reported under "q32". Inputs are seeded synthetic tensors with the configs'
shapes and distributions (starkv_b200.workload); every step reads a >2 GB cache,
far larger than the 126 MB L2, so no flush is needed between steps. Each step is
captured once in a CUDA graph and replayed, as a serving engine runs the decode
(the line's clocks.mode says so; eager when capture is not possible).

Every default run also measures, in the same line: config 4 (256 mixed-length
sequences, skewed ranks, both formats: "c4"), config 5 (the whole 32-layer model's
decode step in a CUDA graph, K/V factors loaded from a synthetic fused_weights.pt:
"model") and, on one GPU, the reference's own Triton decode on the same inputs
("gpu_bar"). --skip heads,c4,model,bar leaves parts out.

N > 1 (torchrun), --parallel context (default): the one 64-sequence batch is split
over the GPUs (strong scaling): every rank decodes all heads over its share of each
sequence's 256-token tiles, and the partials are combined exactly with one NCCL
all-gather and a native kernel (starkv_b200.context_parallel); each GPU reads 1/N
of the K and V codes. Beside it the line reports "heads": the same batch with heads
sharded tensor-parallel (LPT on K width), the north star's split, which keeps the V
codes whole on every rank (the shared latent is read by every head) and so scales
sub-linearly. --parallel seqs gives every GPU its own batch of 64 sequences with no
collective (weak scaling). The step time is always the max over ranks.

--impl reference: the reference's own PyTorch CPU decode math (model.py, imported
from the installed reference in baseline/_ref; the numpy restatement in oracle/
when it is not installed), timed on this host's cores on a bounded sample of the
same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
CLOCKS_DIR = os.environ.get("STARKV_CLOCKS_DIR", os.path.join(ROOT, "clocks"))
sys.path.insert(0, os.path.join(ROOT, "star-kv-serve_b200"))

METRIC = "low-rank paged decode attn µs/layer & HBM GB/s; decode tok/s at 1/2/4/8 B200"
UNIT = "decode tok/s per layer-step"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clock and clock-event reasons sampled through NVML by a thread, every
    millisecond, for as long as the timed region runs (the region is tens of
    milliseconds, shorter than nvidia-smi's start-up). Samples are also written to
    clocks_gpu<i>.csv in the run's output folder (CLOCKS_DIR) as a record."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device):
        import threading
        self.samples, self.err = [], None
        self.path = os.path.join(CLOCKS_DIR, f"clocks_gpu{device.index or 0}.csv")
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            try:
                p = torch_props(device)
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                self.h = N.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = N.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM))
        except Exception as e:   # no NVML: reported, not fatal
            self.err = f"nvml unavailable: {type(e).__name__}"
            return
        self.stop_ev = threading.Event()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        N = self.N
        get_r = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            N.nvmlDeviceGetCurrentClocksThrottleReasons
        while True:
            try:
                self.samples.append((time.perf_counter(), float(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)),
                                     int(get_r(self.h))))
            except Exception as e:
                self.err = f"nvml query failed: {type(e).__name__}"
                return
            if self.stop_ev.wait(0.001):
                return

    def stop(self):
        if self.err and not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err], "samples": 0}
        self.stop_ev.set()
        self.t.join(timeout=5)
        reasons = sorted({nm for _, _, r in self.samples for nm, bit in self.REASONS.items() if r & bit})
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            with open(self.path, "w") as f:
                f.write("t_s,sm_mhz,event_reasons\n")
                t0 = self.samples[0][0] if self.samples else 0.0
                for t, mhz, r in self.samples:
                    f.write(f"{t - t0:.4f},{mhz:.0f},0x{r:x}\n")
        except OSError:
            pass
        sm = [m for _, m, _ in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "source": "nvml, 1 ms"}


def torch_props(device):
    import torch
    return torch.cuda.get_device_properties(device)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def shard_layer_spec(ranks, world, rank):
    from starkv_b200.sharding import lpt_shard
    return lpt_shard(ranks, world)[rank]


def build_layer(quant: bool, world: int, rank: int, device, batch=None, context=None, parallel="context",
                mixed=False):
    from starkv_b200.workload import make_layer, sample_ranks
    if mixed:
        # config 4: a serving batch of 256 sequences with contexts uniform in
        # [1024, 32768] and skewed per-head ranks (K 16..128, V 32..128), seeded
        import numpy as np
        rng = np.random.default_rng(4)
        n = batch or 256
        lens = [int(x) for x in rng.integers(1024, (context or 32768) + 1, size=n)]
        ranks, rv = sample_ranks(32, 4, skewed=True)
    else:
        n, L = (64, 16384) if quant else (64, 8192)
        n, L = batch or n, context or L
        lens = [L] * n
        ranks, rv = sample_ranks(32, 0)
    # sequence split: every rank holds the whole layer and its own batch; context
    # split: every rank holds the whole layer (all heads) and decodes its share of
    # each sequence; head split: each rank holds its heads (LPT)
    heads = list(range(32)) if world == 1 or parallel != "heads" else shard_layer_spec(ranks, world, rank)
    local = [ranks[h] for h in heads]
    layer = make_layer(lens, num_heads=len(local), quant=quant, seed=0, device=device, ranks=local, v_rank=rv)
    return layer, heads


def run_step_fns(layer, device, cp=None):
    import torch
    from starkv_b200.kernels import paged_quant as pq
    from starkv_b200.kernels.paged_decode import paged_starkv_decode, write_kv_bf16
    from starkv_b200 import workspace
    g = torch.Generator(device=device).manual_seed(123)
    n = layer.n
    k_new = torch.randn(n, layer.k_width, generator=g, device=device).to(torch.bfloat16)
    v_new = torch.randn(n, layer.v_rank, generator=g, device=device).to(torch.bfloat16)
    for r, o in zip(layer.ranks, layer.offsets):
        w = -(-r // 16) * 16
        k_new[:, o + r:o + w] = 0
    # the new token of sequence b sits at position L_b - 1
    pos = torch.tensor([L - 1 for L in layer.seq_lens_host], device=device)
    slots = (layer.block_table[torch.arange(n, device=device), pos // 16].long() * 16 + pos % 16)
    H = layer.num_heads
    ws = workspace.reserve(device, n, H, len(layer.ranks), layer.k_width, layer.v_rank, layer.max_seq_len)
    out = torch.empty(n, H, 128, dtype=torch.bfloat16, device=device)
    part = torch.empty(n * H * 130, dtype=torch.float32, device=device) if cp else None
    # context split: the new token of every sequence lies in the last rank's share
    writes = cp is None or cp[0] == cp[1] - 1
    if cp is not None:
        from starkv_b200.context_parallel import combine

    def step(q=None, kn=None, vn=None, bt=None, sl=None):
        q = layer.query if q is None else q
        kn = k_new if kn is None else kn
        vn = v_new if vn is None else vn
        bt = layer.block_table if bt is None else bt
        sl = layer.seq_lens if sl is None else sl
        if layer.quant:
            if writes:
                pq.pack_kv(kn, vn, layer.kv_cache, slots, layer.row, layer.k_ranks, layer.k_head_offsets,
                           layer.k_nouts)
            r = pq.paged_quant_decode(q, layer.kv_cache, bt, sl, layer.max_seq_len, layer.row, layer.k_up,
                                      layer.head_of_lane, layer.k_tiles, layer.v_up_by_q, layer.cos_sin_cache,
                                      layer.scale, out=out, ws=ws, context=cp, partial=part)
        else:
            if writes:
                write_kv_bf16(kn, vn, layer.kv_cache, slots)
            r = paged_starkv_decode(q, layer.kv_cache, bt, sl, layer.max_seq_len, layer.k_up, layer.k_ranks,
                                    layer.k_head_offsets, layer.k_width, layer.v_up_by_q, layer.cos_sin_cache,
                                    layer.scale, out=out, ws=ws, context=cp, partial=part)
        return combine(*r, result=out) if cp is not None else r
    return step, (k_new, v_new)


def measure(layer, device, steps, warmup, dist_on, cp=None):
    import ctypes as C
    import torch
    import torch.distributed as dist
    from starkv_b200 import _lib
    step, (k_new, v_new) = run_step_fns(layer, device, cp)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    graphs = []   # released before returning (they may hold NCCL calls)

    def graphed(fn):
        """fn captured in a CUDA graph (the decode path allocates and synchronises
        nothing, so it captures as a serving engine runs it); eager if capture fails."""
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            torch.cuda.synchronize()
            graphs.append(g)
            return g.replay, "cuda graph"
        except Exception as e:   # noqa: BLE001 - recorded in the line, timed eagerly
            torch.cuda.synchronize()
            return fn, f"eager (capture failed: {type(e).__name__})"

    def timed(fn, k):
        if dist_on:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(k):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / k
        if dist_on:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    run, mode = graphed(step)
    for _ in range(2):
        run()
    clk = Clocks(device)
    ms = timed(run, steps)
    clocks = clk.stop()
    clocks["mode"] = mode

    # per-kernel durations, live CUDA events on the launching stream (separate pass)
    lib = _lib.lib()
    lib.starkv_profile_begin(steps)
    for _ in range(steps):
        step()
    torch.cuda.synchronize()
    kms = (C.c_float * 4)()
    ncalls = C.c_int32(0)
    _lib.check(lib.starkv_profile_end(kms, C.byref(ncalls)), "profile")
    per_kernel = [kms[i] / max(ncalls.value, 1) for i in range(4)]

    # end to end through the public API with host buffers (pinned), H2D inputs + D2H output
    n, H = layer.n, layer.num_heads
    hq = layer.query.cpu().pin_memory()
    hk, hv = k_new.cpu().pin_memory(), v_new.cpu().pin_memory()
    hbt = layer.block_table.cpu().pin_memory()
    hsl = layer.seq_lens.cpu().pin_memory()
    dq, dk, dv = torch.empty_like(layer.query), torch.empty_like(k_new), torch.empty_like(v_new)
    dbt, dsl = torch.empty_like(layer.block_table), torch.empty_like(layer.seq_lens)
    hout = torch.empty(n, H, 128, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        dbt.copy_(hbt, non_blocking=True)
        dsl.copy_(hsl, non_blocking=True)
        o = step(dq, dk, dv, dbt, dsl)
        hout.copy_(o, non_blocking=True)
    for _ in range(2):
        e2e_step()
    e2e_run, _ = graphed(e2e_step)
    for _ in range(2):
        e2e_run()
    e2e_ms = timed(e2e_run, steps)
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hbt, hsl))
    d2h = hout.numel() * hout.element_size()
    last = step()
    torch.cuda.synchronize()
    graphs.clear()
    return ms, per_kernel, clocks, e2e_ms, h2d, d2h, last


def layer_case(args, device, world, rank, dist_on):
    """One whole compressed attention layer per step (starkv_b200.layer): Q / kv_down
    / o_proj GEMMs, rotary, cache write or pack, paged decode; hidden 4096, 32 heads,
    config 2 (bf16) and config 3 (3.2-bit) caches. N > 1: heads sharded (LPT) with the
    o_proj all-reduce, or (seqs) a batch per GPU."""
    import torch
    import torch.distributed as dist
    from starkv_b200 import layer as Ly
    from starkv_b200 import workspace
    from starkv_b200.workload import make_layer, rope_cos_sin, sample_ranks
    tp = world if dist_on and args.parallel == "heads" else 1
    out = {}
    for quant in (False, True):
        n, L = (64, 16384) if quant else (64, 8192)
        n, L = args.batch or n, args.context or L
        ranks, rv = sample_ranks(32, 0)
        w = Ly.random_weights(4096, 32, ranks, rv, seed=0, device=device)
        ly = Ly.StarKVAttentionLayer(w, rope_cos_sin(L, device), quant=quant, rank=rank if tp > 1 else 0,
                                     world=tp)
        del w
        cl = make_layer([L] * n, num_heads=ly.num_heads, quant=quant, seed=0, device=device,
                        ranks=ly.k_ranks_host, v_rank=rv)
        g = torch.Generator(device=device).manual_seed(7)
        hidden = torch.randn(n, 4096, generator=g, device=device).to(torch.bfloat16)
        pos = torch.full((n,), L - 1, device=device)
        slots = cl.block_table[torch.arange(n, device=device), pos // 16].long() * 16 + pos % 16
        ws = workspace.reserve(device, n, ly.num_heads, ly.num_kv_heads, ly.k_width, rv, cl.max_seq_len)

        def fn():
            return ly.forward(hidden, pos, cl.kv_cache, cl.block_table, cl.seq_lens, cl.max_seq_len, slots, ws=ws)

        for _ in range(args.warmup):
            fn()
        if dist_on:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        if dist_on:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        reps = world if dist_on and args.parallel == "seqs" else 1
        out["q32" if quant else "bf16"] = {"us_per_layer": round(ms * 1e3, 1), "ms_per_step": round(ms, 4),
                                          "value": round(reps * n / (ms * 1e-3), 1), "unit": UNIT,
                                          "batch": n, "context": L, "heads_per_gpu": ly.num_heads,
                                          "k_width": ly.k_width, "v_rank": rv}
        del ly, cl, ws
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({"case": "layer", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "parallelism": ("single" if world == 1 else f"tp{world} (heads, LPT, o_proj all-reduce)"
                                          if tp > 1 else f"dp{world} (sequences, a batch per GPU)"),
                          "hidden": 4096, "heads": 32, **out}), flush=True)


def model_case(args, device, world, rank, dist_on):
    """Config 5: decode step of the whole 32-layer Llama-2-7B-geometry model
    (starkv_b200.model; layers 0, 1, 2, 31 full-rank, the rest STAR-KV at
    comp-ratio 0.75), `--batch` sessions at context `--context` (default 32768),
    tensor parallel over the N GPUs with the o_proj / down_proj all-reduces; caches
    filled with synthetic values. Without `--batch` the sessions are as many as fit in
    85% of the HBM left free after the weights (the configuration's "max concurrency").
    With `--parallel context` the compressed layers split their caches by pages instead
    of heads (page p of a sequence on rank p % N; every rank decodes all heads over its
    pages, and the partials are all-gathered and combined exactly). The step is captured
    in a CUDA graph when capture works, else run eagerly."""
    line = model_measure(args, device, world, rank, dist_on, args.parallel, args.batch, args.context)
    if rank == 0:
        print(json.dumps({"case": "model", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, **line}),
              flush=True)


def synthetic_checkpoint_path(cfg, dist_on, rank):
    """Write config 5's random-init fused_weights.pt (the reference layout,
    starkv_b200.checkpoint) once per job into a temporary folder; every rank then
    loads it. Returns the path (the caller removes it after loading)."""
    import tempfile
    import torch.distributed as dist
    from starkv_b200.checkpoint import write_synthetic_checkpoint
    from starkv_b200.model import checkpoint_layer_ranks
    port = os.environ.get("MASTER_PORT", "single")
    path = os.path.join(tempfile.gettempdir(), f"starkv_config5_fused_weights_{port}_{os.getuid()}.pt")
    if rank == 0:
        write_synthetic_checkpoint(path, checkpoint_layer_ranks(cfg), cfg.hidden, cfg.heads, seed=cfg.seed)
    if dist_on:
        dist.barrier()
    return path


def model_measure(args, device, world, rank, dist_on, parallel, batch=None, context=None):
    """Config 5 decode step (see model_case); returns the measurement as a dict."""
    import torch
    import torch.distributed as dist
    from starkv_b200 import context_parallel as cp
    from starkv_b200.model import ModelConfig, StarKVModel
    C = context or 32768
    split = "context" if dist_on and parallel == "context" else "heads"
    cfg = ModelConfig(max_pos=C)
    ckpt = None
    if args.model_weights == "checkpoint":
        ckpt = synthetic_checkpoint_path(cfg, dist_on, rank)
    model = StarKVModel(cfg, device, quant=False, rank=rank if dist_on else 0, world=world if dist_on else 1,
                        group=None, attn_parallel=split, checkpoint=ckpt)
    if ckpt is not None:
        if dist_on:
            dist.barrier()
        if rank == 0:
            os.remove(ckpt)
    if batch:
        n = args.batch
    else:
        free = torch.cuda.mem_get_info(device)[0]
        n = max(1, int(0.85 * free / (C * model.kv_bytes_per_token())))
        if dist_on:   # every rank runs the same sessions
            t = torch.tensor([n], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            n = int(t.item())
    pages = -(-C // 16)
    local = None
    if split == "context":
        # this rank's pages of every sequence, as its own local sequences
        llen = int(cp.local_len(C, rank, world))
        lpages = max(-(-llen // 16), 1)
        lbt = (torch.randperm(n * lpages, generator=torch.Generator().manual_seed(2 + rank)) + 1).view(n, lpages)
        lbt = lbt.to(device=device, dtype=torch.int32)
        li = int(cp.local_index(C - 1, world))
        if int(cp.page_owner(C - 1, world)) == rank:
            lslots = lbt[:, li // 16].long() * 16 + li % 16
        else:
            lslots = torch.full((n,), -1, dtype=torch.long, device=device)
        local = (lbt, torch.full((n,), llen, dtype=torch.int32, device=device), max(llen, 1), lslots)
        caches = model.allocate_caches(n * pages + 1, n * lpages + 1)
    else:
        caches = model.allocate_caches(n * pages + 1)
    g = torch.Generator(device=device).manual_seed(3)
    for c in caches:
        for t in (c if isinstance(c, tuple) else (c,)):
            t.normal_(0.0, 1.0, generator=g)
    perm = torch.randperm(n * pages, generator=torch.Generator().manual_seed(1)) + 1
    bt = perm.view(n, pages).to(device=device, dtype=torch.int32)
    pos = torch.full((n,), C - 1, device=device)
    slots = bt[torch.arange(n, device=device), pos // 16].long() * 16 + pos % 16
    seq_lens = torch.full((n,), C, dtype=torch.int32, device=device)
    tokens = torch.randint(0, cfg.vocab, (n,), generator=g, device=device)

    def step():
        return model.decode_step(tokens, pos, caches, bt, seq_lens, C, slots, local=local)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    graph, mode = None, "eager"
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
        mode = "cuda graph"
    except Exception as e:   # capture unsupported somewhere: time the eager step
        graph = None
        mode = f"eager (capture failed: {type(e).__name__})"
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step
    for _ in range(2):
        run()
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if dist_on:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    kv_gb = sum(sum(t.numel() * t.element_size() for t in (c if isinstance(c, tuple) else (c,))) for c in caches) / 1e9
    del graph, model, caches
    torch.cuda.empty_cache()
    return {"workload": "config5: 32-layer Llama-2-7B geometry (hidden 4096, FFN 11008, vocab 32000), layers "
                        "0,1,2,31 full-rank bf16 KV, 28 STAR-KV bf16 layers at comp-ratio 0.75",
            "weights": ("K/V factors from a synthetic fused_weights.pt (reference layout, random init) through "
                        "starkv_b200.checkpoint; other weights seeded random-init" if ckpt is not None
                        else "seeded random-init"),
            "sessions": n, "context": C, "parallelism": f"tp{world}" if dist_on else "single",
            "compressed_attention_split": "pages (context parallel)" if split == "context" else "heads",
            "mode": mode, "ms_per_step": round(ms, 3), "value": round(n / (ms * 1e-3), 1),
            "unit": "decode tok/s (whole model)", "kv_cache_gb_per_gpu": round(kv_gb, 1),
            "data": "synthetic (seeded caches)"}


def prefill_measure(device, steps, warmup, tf_peak, peak_kind):
    """Dense prefill attention (the reference prefill's flash_attn_varlen_func,
    attention.py:246-250) on the library's kernel: 8 prompts x 2048 tokens, 32 heads
    x 128, bf16, causal; beside it the same call through flash_attn (the reference's
    library) and torch SDPA when they run here."""
    import torch
    from starkv_b200.kernels.prefill import cu_seqlens_of, prefill_attention
    lens, H = [2048] * 8, 32
    T = sum(lens)
    g = torch.Generator(device=device).manual_seed(7)
    q, k, v = (torch.randn(T, H, 128, generator=g, device=device).to(torch.bfloat16) for _ in range(3))
    cu = cu_seqlens_of(lens, device)
    scale = 128 ** -0.5
    flops = 4 * 128 * H * sum(L * (L + 1) // 2 for L in lens)
    out = torch.empty_like(q)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    ms = timed(lambda: prefill_attention(q, k, v, lens, scale, cu_seqlens=cu, out=out))
    res = {"workload": "dense prefill attention: 8 prompts x 2048 tokens, 32 heads x 128, bf16, causal",
           "ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
           "roofline": {"bound": "tensor", "achieved": round(flops / (ms * 1e-3) / 1e12, 1), "peak": tf_peak,
                        "unit": "TFLOP/s", "frac": round(flops / (ms * 1e-3) / 1e12 / tf_peak, 4),
                        "peak_kind": peak_kind},
           "l2": "inputs 100 MB; compute-bound"}
    try:
        from flash_attn import flash_attn_varlen_func
        fa = timed(lambda: flash_attn_varlen_func(q, k, v, cu, cu, 2048, 2048, softmax_scale=scale, causal=True))
        res["flash_attn_ms"] = round(fa, 4)
    except Exception as e:   # noqa: BLE001 - the comparison is optional
        res["flash_attn_ms"] = f"unavailable: {type(e).__name__}"
    try:
        qs, ks, vs = (x.view(8, 2048, H, 128).transpose(1, 2) for x in (q, k, v))
        sd = timed(lambda: torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=scale))
        res["torch_sdpa_ms"] = round(sd, 4)
    except Exception as e:   # noqa: BLE001
        res["torch_sdpa_ms"] = f"unavailable: {type(e).__name__}"
    return res


def rank_tokens(layer, cp):
    """Tokens this rank decodes: all, or its share of each sequence's 256-token tiles."""
    if cp is None:
        return layer.kv_tokens()
    r, w = cp
    tot = 0
    for L in layer.seq_lens_host:
        T = -(-L // 256)
        tot += max(0, min(256 * (T * (r + 1) // w), L) - 256 * (T * r // w))
    return tot


# DRAM traffic / algorithmic bytes of each kernel, from one ncu capture per kernel at
# batch 16 with the config shapes (dram__bytes_read.sum + dram__bytes_write.sum;
# profiles/scores_pv_pvq_kernels_batch16.md). Both grow with the tokens processed, so
# a full launch's traffic is its algorithmic bytes times this ratio.
TRAFFIC_RATIO = {(False, "scores"): 414.386944 / 364.904448, (False, "pv"): 444.123136 / 402.653184,
                 (True, "scores"): 280.232960 / 216.006656, (True, "pv"): 283.142400 / 202.637312}


def roofline_for(layer, per_kernel, hbm_peak, cp=None):
    """Dominant kernel's algorithmic bytes per launch / its event-timed duration."""
    T = rank_tokens(layer, cp)
    names = ["fold", "scores", "pv", "lift"]
    k = max(range(4), key=lambda i: per_kernel[i])
    if layer.quant:
        per_tok = {1: layer.k_width // 2 + 4 * len(layer.ranks), 2: 4 + layer.row.v_bytes}
    else:
        per_tok = {1: 2 * layer.k_width, 2: 2 * layer.v_rank}
    alg = T * per_tok.get(k, 0)
    ms = per_kernel[k]
    achieved = alg / (ms * 1e-3) / 1e9 if ms > 0 else 0.0
    ratio = TRAFFIC_RATIO.get((layer.quant, names[k]))
    return {"kernel": names[k], "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
            "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
            "traffic": int(alg * ratio) if ratio else None,
            "traffic_source": "ncu DRAM bytes at batch 16, scaled by tokens per launch" if ratio else None,
            "alg_bytes_per_launch": alg, "ms_per_launch": round(ms, 4),
            "kernel_ms": {nm: round(v, 4) for nm, v in zip(names, per_kernel)}}


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def triton_bar(layer, device, steps, ours_decode_ms, ours_out=None):
    """The reference's own GPU decode on the same inputs: paged_starkv_decode
    (paged_decode.py:150-226) or paged_quant_decode (paged_quant.py:357-411), imported
    unmodified from the installed reference (baseline/_ref) and JIT-compiled by this
    box's Triton. Timed with CUDA events after a warm-up that includes compilation;
    decode only (no cache write), beside our decode-only time (sum of our 4 kernels).
    The output is compared with ours as a sanity check (max abs difference)."""
    import torch
    if not os.path.isdir(os.path.join(REF_DIR, "starkv_serve")):
        return {"unavailable": "reference not installed in baseline/_ref"}
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        from starkv_serve.kernels import paged_decode as rpd
        from starkv_serve.kernels import paged_quant as rpq
    except Exception as e:   # noqa: BLE001 - reported, not fatal
        return {"unavailable": f"import failed: {type(e).__name__}: {e}"[:300]}
    L = layer
    if L.quant:
        row = rpq.QuantRow(L.k_width, len(L.ranks), L.v_rank)
        _, hol, tiles = rpq.k_tables(L.ranks, device)

        def fn():
            return rpq.paged_quant_decode(L.query, L.kv_cache, L.block_table, L.seq_lens, L.max_seq_len, row,
                                          L.k_up, hol, tiles, L.v_up_by_q, L.cos_sin_cache, L.scale)
    else:
        def fn():
            return rpd.paged_starkv_decode(L.query, L.kv_cache, L.block_table, L.seq_lens, L.max_seq_len, L.k_up,
                                           L.k_ranks, L.k_head_offsets, L.k_width, L.v_up_by_q, L.cos_sin_cache,
                                           L.scale)
    try:
        t0 = time.perf_counter()
        out = fn()
        torch.cuda.synchronize()
        compile_s = time.perf_counter() - t0
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
    except Exception as e:   # noqa: BLE001 - a compile or launch failure is the result
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    res = {"impl": "reference Triton (baseline/_ref, unmodified), this box's Triton JIT",
           "ms_per_decode": round(ms, 4), "ours_decode_ms": round(ours_decode_ms, 4),
           "speedup": round(ms / ours_decode_ms, 3) if ours_decode_ms > 0 else None,
           "first_call_s": round(compile_s, 2), "steps": steps}
    if ours_out is not None:
        res["max_abs_diff_vs_ours"] = float((out.float() - ours_out.float()).abs().max())
    return res


def reference_torch_decode():
    """The reference's own PyTorch CPU decode math, imported unmodified from the
    installed reference (baseline/_ref): model._expand_ragged_k (model.py:1204-1220),
    model._rope_tables (model.py:127-137) and transformers' rotate_half, composed
    as the no-Triton decode branch does (model.py:1333-1386): expand K per head
    from its rank, rotate it, q.K^T * scale, softmax in the cache dtype, P.V over
    the shared V codes, bmm lift per query head. None when not importable."""
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import torch
        import torch.nn.functional as F
        import model as ref_model
    except Exception:   # noqa: BLE001 - the numpy port is the fallback
        return None

    def decode(q, key_states, value_states, k_up, segments, u_by_q, inv_freq, scale):
        # q [B, Hq, 1, Hd]; key_states rank-major [B, W, L]; value_states [B, L, rv]
        key_full = ref_model._expand_ragged_k(key_states, k_up, segments)
        k_cos, k_sin = ref_model._rope_tables(inv_freq, key_full.shape[-2], key_full.device, key_full.dtype)
        key_full = key_full * k_cos + ref_model.rotate_half(key_full) * k_sin
        attn = torch.matmul(q, key_full.transpose(2, 3)) * scale
        attn = F.softmax(attn, dim=-1).to(q.dtype)
        prob_v = attn.squeeze(2) @ value_states
        return torch.bmm(prob_v.transpose(0, 1), u_by_q).transpose(0, 1)
    return decode


def reference_cpu_time(batch, L, dtype_name, seconds=10.0, reps_min=3):
    """Time the reference's CPU decode (reference_torch_decode) on `batch` sequences
    of `L` tokens (contiguous cache, config-1 sampling: K ranks {16,32,48,64}, V
    {32,64} per head, codes and q ~ N(0,1), B_k / B_v ~ N(0, 1/sqrt(rank))) with
    all host threads. Returns (sequences per second, ms per call) or None."""
    import torch
    dec = reference_torch_decode()
    if dec is None:
        return None
    torch.set_num_threads(os.cpu_count())
    key = (batch, L, dtype_name)
    if key not in _REF_INPUTS:
        _REF_INPUTS[key] = _reference_inputs(batch, L, dtype_name)
    q, ks, vs, k_up, seg, u_by_q, inv_freq = _REF_INPUTS[key]
    dec(q, ks, vs, k_up, seg, u_by_q, inv_freq, 128 ** -0.5)   # warm-up
    times, t_all = [], time.perf_counter()
    while len(times) < reps_min or (time.perf_counter() - t_all < seconds and len(times) < 50):
        t0 = time.perf_counter()
        dec(q, ks, vs, k_up, seg, u_by_q, inv_freq, 128 ** -0.5)
        times.append(time.perf_counter() - t0)
    ms = statistics.median(times) * 1e3
    return batch / (ms * 1e-3), ms


_REF_INPUTS = {}


def _reference_inputs(batch, L, dtype_name):
    import torch
    from starkv_b200.workload import sample_ranks
    dt = {"fp32": torch.float32, "bf16": torch.bfloat16}[dtype_name]
    g = torch.Generator().manual_seed(0)
    ranks, rv = sample_ranks(32, 0)
    widths = [-(-r // 16) * 16 for r in ranks]
    offsets = [sum(widths[:h]) for h in range(32)]
    W = sum(widths)
    k_up = torch.zeros(W, 128)
    for r, o in zip(ranks, offsets):
        k_up[o:o + r] = torch.randn(r, 128, generator=g) / r ** 0.5
    key_states = torch.randn(batch, W, L, generator=g)
    for r, o, w in zip(ranks, offsets, widths):
        key_states[:, o + r:o + w] = 0
    value_states = torch.randn(batch, L, rv, generator=g)
    u_by_q = torch.randn(32, rv, 128, generator=g) / rv ** 0.5
    q = torch.randn(batch, 32, 1, 128, generator=g)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    return (q.to(dt), key_states.to(dt), value_states.to(dt), k_up.to(dt), list(zip(offsets, ranks)), u_by_q.to(dt),
            inv_freq)


def cpu_baseline_line(seconds=10.0):
    """cpu_baseline of the JSON line: the reference's own torch CPU math on a sample of
    config 2 (4 of its 64 sequences, 8192 tokens, bf16 as the cache is), plus
    BASELINE config 1 (batch 4, context 2048) in fp32 and bf16; the numpy oracle port
    when the reference is not importable."""
    main = reference_cpu_time(4, 8192, "bf16", seconds)
    if main is None:
        rate, desc = cpu_sample_time(False)
        return {"value": round(rate, 3), "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": desc}
    c1 = {dt: reference_cpu_time(4, 2048, dt, seconds=3.0, reps_min=5) for dt in ("fp32", "bf16")}
    return {"value": round(main[0], 3), "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
            "sample": "4 of config 2's sequences x 8192 tokens per call, bf16, the reference's own torch CPU "
                      "decode (model.py _expand_ragged_k / _rope_tables / no-Triton branch) from baseline/_ref",
            "ms_per_call": round(main[1], 2),
            "config1_ms": {dt: (round(v[1], 2) if v else None) for dt, v in c1.items()},
            "config1": "batch 4 x 2048 tokens, 32 heads, contiguous cache, median of >= 5 after 1 warm-up"}


def cpu_sample_time(quant: bool, seconds: float = 12.0):
    """Reference algorithm (oracle port, numpy, all host cores) on whole sequences of
    the same workload; returns (sequences per second, sample description)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import starkv_oracle as O
    from starkv_b200.workload import sample_ranks
    rng = np.random.default_rng(0)
    ranks, rv = sample_ranks(32, 0)
    widths, offsets, W = O.k_layout(ranks)
    L = 16384 if quant else 8192
    H = 32
    q = rng.standard_normal((H, 128), dtype=np.float32)
    k_up = np.zeros((W, 128), np.float32)
    for r, o in zip(ranks, offsets):
        k_up[o:o + r] = rng.standard_normal((r, 128), dtype=np.float32) / np.sqrt(r)
    v_up = rng.standard_normal((H, rv, 128), dtype=np.float32) / np.sqrt(rv)
    cs = O.rope_cos_sin(L)
    row = O.QuantRow(W, H, rv)
    if quant:
        rows = O.pack_rows(rng.standard_normal((L, W), dtype=np.float32),
                           rng.standard_normal((L, rv), dtype=np.float32), row, ranks)
    else:
        kc = rng.standard_normal((L, W), dtype=np.float32)
        vc = rng.standard_normal((L, rv), dtype=np.float32)
    done, t0 = 0, time.perf_counter()
    while True:
        if quant:
            kd, vd = O.unpack_rows(rows, row, ranks)
            O.attend_one(q, kd, vd, k_up, ranks, offsets, 1, v_up, cs, 128 ** -0.5, dtype=np.float32)
        else:
            O.attend_one(q, kc, vc, k_up, ranks, offsets, 1, v_up, cs, 128 ** -0.5, dtype=np.float32)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 64:
            break
    return done / el, f"{done} sequence(s) x {L} tokens, 32 heads, float32 numpy (oracle port)"


def ours(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist_on = world > 1
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if dist_on:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))
    hbm_peak, tf_peak, peak_kind = peaks()
    if args.case in ("layer", "model"):
        (layer_case if args.case == "layer" else model_case)(args, device, world, rank, dist_on)
        if dist_on:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == "prefill":
        if rank == 0:
            print(json.dumps({"case": "prefill", **prefill_measure(device, args.steps, args.warmup, tf_peak,
                                                                   peak_kind)}), flush=True)
    elif args.case == "c4":
        # config 4 alone (mixed lengths, skewed ranks), both formats: one line, no baselines
        c4 = {key: decode_case(quant, True, args, world, rank, device, dist_on, hbm_peak)
              for quant, key in ((False, "bf16"), (True, "q32"))}
        if rank == 0:
            print(json.dumps({"case": "c4", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                              **c4_summary(c4, args.parallel, world, hbm_peak)}), flush=True)
    elif args.case in ("c2", "c3"):
        # single-configuration run (profiling): short line, no baselines
        r = decode_case(args.case == "c3", False, args, world, rank, device, dist_on, hbm_peak,
                        bar=world == 1 and "bar" not in args.skip)
        if rank == 0:
            print(json.dumps({"case": args.case, "batch": r["n"], "context": r["context"],
                              "ms_per_step": round(r["ms"], 4), "kernel_ms": r["roof"]["kernel_ms"],
                              "hbm_gbs": round(r["alg"] / (r["ms"] * 1e-3) / 1e9, 1),
                              "roofline_frac": r["roof"]["frac"], "gpu_bar": r.get("bar")}), flush=True)
    else:
        bar = world == 1 and "bar" not in args.skip
        b = decode_case(False, False, args, world, rank, device, dist_on, hbm_peak, bar=bar)
        q = decode_case(True, False, args, world, rank, device, dist_on, hbm_peak, bar=bar)
        heads = None
        if dist_on and args.parallel != "heads" and "heads" not in args.skip:
            heads = decode_case(False, False, args, world, rank, device, dist_on, hbm_peak, parallel="heads")
        c4 = None
        if "c4" not in args.skip:
            c4 = {key: decode_case(quant, True, args, world, rank, device, dist_on, hbm_peak)
                  for quant, key in ((False, "bf16"), (True, "q32"))}
        model = None
        if "model" not in args.skip:
            model = model_measure(args, device, world, rank, dist_on, args.parallel)
        prefill = None
        if world == 1 and "prefill" not in args.skip:
            prefill = prefill_measure(device, max(args.steps, 5), max(args.warmup, 3), tf_peak, peak_kind)
        if rank == 0:
            reps = world if dist_on and args.parallel == "seqs" else 1   # batches in the job (seqs: one per GPU)
            cpu_line = cpu_baseline_line() if world == 1 else None
            par = ("single" if world == 1 else f"dp{world} (sequences: 64 per GPU, no collective)"
                   if args.parallel == "seqs" else f"cp{world} (context split, all heads per GPU)"
                   if args.parallel == "context" else f"tp{world} (heads, LPT by K width)")
            cp_on = dist_on and args.parallel == "context"
            line = {
                "metric": METRIC, "value": round(reps * b["n"] / (b["ms"] * 1e-3), 1), "unit": UNIT,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(b["ms"], 4), "us_per_layer": round(b["ms"] * 1e3, 1),
                "hbm_gbs": round(reps * b["alg"] / (b["ms"] * 1e-3) / 1e9, 1),
                "hbm_frac_step": round(reps * b["alg"] / (b["ms"] * 1e-3) / 1e9 / (hbm_peak * world), 4),
                "higher_is_better": True, "scaling": "strong" if dist_on and args.parallel != "seqs" else "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, config shapes)",
                "config": {"workload": "config2: paged bf16 low-rank decode, 1 layer, 64 seqs x 8192 tokens, "
                                       "32 heads x 128, page 16, cache write + decode per step",
                           "batch": 64, "global_batch": 64 * reps, "context": 8192,
                           "heads_per_gpu": 32 if not dist_on or args.parallel != "heads" else 32 // world,
                           "parallelism": par, "l2": "inputs (2.9 GB cache) larger than L2; no flush"},
                "roofline": dict(b["roof"], peak_kind=peak_kind),
                "e2e": {"value": round(reps * b["n"] / (b["e2e_ms"] * 1e-3), 1), "unit": UNIT,
                        "h2d_bytes_per_step": b["h2d"], "d2h_bytes_per_step": b["d2h"],
                        "ms_per_step": round(b["e2e_ms"], 4)},
                "gpu_bar": {"bf16": b.get("bar"), "q32": q.get("bar")} if bar else None,
                # our kernels per step on rank 0: fold, scores, P.V, lift, the cache write (the
                # writing rank: all of them, or under the context split the last one), the combine
                "gpu_launches": (4 + (0 if cp_on and world > 1 else 1) + (1 if cp_on else 0)) * args.steps,
                "clocks": b["clocks"],
                "q32": dict(step_summary(q, reps, world, hbm_peak, peak_kind),
                            workload="config3: 3.2-bit paged decode, 64 seqs x 16384 tokens, pack + decode per step",
                            tflops=round(reps * q["flops"] / (q["ms"] * 1e-3) / 1e12, 1)),
            }
            if heads is not None:
                line["heads"] = dict(step_summary(heads, 1, world, hbm_peak, peak_kind),
                                     workload="config2 with heads sharded tensor-parallel (LPT by K width); "
                                              "the V latent is read whole on every rank", heads_per_gpu=32 // world)
            if c4 is not None:
                line["c4"] = c4_summary(c4, args.parallel, world, hbm_peak)
            if model is not None:
                line["model"] = model
            if prefill is not None:
                line["prefill"] = prefill
            if cpu_line is not None:
                line["cpu_baseline"] = cpu_line
            print(json.dumps(line), flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


def decode_case(quant, mixed, args, world, rank, device, dist_on, hbm_peak, bar=False, parallel=None):
    """Build one configuration's layer (config 2 / 3, or config 4 when `mixed`),
    time its step (`measure`) and, with `bar`, the reference's Triton decode on the
    same inputs; returns the figures (the layer itself is freed)."""
    import torch
    parallel = parallel or args.parallel
    batch, context = (None, None) if mixed else (args.batch, args.context)
    layer, _ = build_layer(quant, world, rank, device, batch, context, parallel, mixed=mixed)
    cp = (rank, world) if dist_on and parallel == "context" else None
    ms, per_kernel, clocks, e2e_ms, h2d, d2h, last = measure(layer, device, args.steps, args.warmup, dist_on, cp)
    r = dict(n=layer.n, context=layer.seq_lens_host[0], tokens=layer.kv_tokens(), k_width=layer.k_width,
             v_rank=layer.v_rank, ms=ms, per_kernel=per_kernel, clocks=clocks, e2e_ms=e2e_ms, h2d=h2d, d2h=d2h,
             alg=layer.algorithmic_bytes(), flops=layer.algorithmic_flops(),
             roof=roofline_for(layer, per_kernel, hbm_peak, cp))
    if bar:
        r["bar"] = triton_bar(layer, device, args.steps, sum(per_kernel), last)
    del last, layer
    torch.cuda.empty_cache()
    return r


def step_summary(r, reps, world, hbm_peak, peak_kind):
    """Sub-object of the JSON line for one measured configuration."""
    return {"value": round(reps * r["n"] / (r["ms"] * 1e-3), 1), "unit": UNIT,
            "ms_per_step": round(r["ms"], 4), "us_per_layer": round(r["ms"] * 1e3, 1),
            "hbm_gbs": round(reps * r["alg"] / (r["ms"] * 1e-3) / 1e9, 1),
            "hbm_frac_step": round(reps * r["alg"] / (r["ms"] * 1e-3) / 1e9 / (hbm_peak * world), 4),
            "roofline": dict(r["roof"], peak_kind=peak_kind), "e2e_ms_per_step": round(r["e2e_ms"], 4),
            "clocks": r["clocks"]}


def c4_summary(c4, parallel, world, hbm_peak):
    """Config 4 (256 mixed-length sequences, skewed ranks), both formats."""
    reps = world if world > 1 and parallel == "seqs" else 1
    out = {"workload": "config4: 256 seqs, contexts seeded uniform in [1024, 32768], skewed ranks (K 16..128, "
                       "V 32..128 per head), 32 heads, cache write / pack + decode per step",
           "parallelism": ("single" if world == 1 else f"dp{world} (sequences, a batch per GPU)"
                           if parallel == "seqs" else f"cp{world} (context split)"
                           if parallel == "context" else f"tp{world} (heads, LPT by rank)"),
           "sequences": c4["bf16"]["n"] * reps, "tokens": int(c4["bf16"]["tokens"])}
    for key, r in c4.items():
        out[key] = {"ms_per_step": round(r["ms"], 4), "value": round(reps * r["n"] / (r["ms"] * 1e-3), 1),
                    "unit": UNIT, "hbm_gbs": round(reps * r["alg"] / (r["ms"] * 1e-3) / 1e9, 1),
                    "hbm_frac_step": round(reps * r["alg"] / (r["ms"] * 1e-3) / 1e9 / (hbm_peak * world), 4),
                    "k_width": r["k_width"], "v_rank": r["v_rank"], "kernel_ms": r["roof"]["kernel_ms"],
                    "clocks": r["clocks"]}
    return out


def reference(args):
    """The reference arm: the reference's own torch CPU decode (reference_torch_decode)
    on this host's cores, each step one call on 4 of config 2's sequences (bf16, 8192
    tokens); the numpy oracle port when the reference is not importable. Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    dec = reference_torch_decode()
    rates, desc, kind, dtype = [], None, "reference", "bf16"
    for i in range(args.warmup + args.steps):
        if dec is not None:
            r = reference_cpu_time(4, 8192, "bf16", seconds=0.0, reps_min=1)[0]
            desc = ("4 of config 2's sequences x 8192 tokens per step, bf16, the reference's own torch CPU decode "
                    f"(model.py _expand_ragged_k / _rope_tables / no-Triton branch), {torch.get_num_threads()} threads")
        else:
            r, desc = cpu_sample_time(False, seconds=2.0)
            kind, dtype = "port", "f32"
        if i >= args.warmup:
            rates.append(r)
    v = statistics.median(rates)
    line = {"metric": METRIC, "value": round(v, 3), "unit": UNIT, "impl": "reference",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": dtype, "data": "synthetic (seeded, config shapes)",
            "config": {"workload": "config2: paged bf16 low-rank decode, 1 layer, 64 seqs x 8192 tokens, "
                                   "32 heads x 128 (CPU: a bounded sample of the sequences per step)"},
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": os.cpu_count(), "kind": kind,
                             "sample": desc},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--case", default="both", choices=["both", "c2", "c3", "c4", "layer", "model", "prefill"],
                    help="c2 / c3 alone: one configuration, short output (profiling)")
    ap.add_argument("--parallel", default="context", choices=["seqs", "context", "heads"],
                    help="N > 1: one batch split over the GPUs by each sequence's tiles (context, default; the "
                         "head split is measured beside it), or by heads; or a batch of sequences per GPU (seqs, "
                         "weak scaling)")
    ap.add_argument("--skip", default="", help="comma list of parts of the default run to leave out: "
                                               "heads, c4, model, bar, prefill")
    ap.add_argument("--model-weights", default="checkpoint", choices=["checkpoint", "random"],
                    help="config 5: K/V factors from a synthetic fused_weights.pt (default) or drawn in place")
    ap.add_argument("--batch", type=int, default=None, help="override the batch (profiling small cases)")
    ap.add_argument("--context", type=int, default=None, help="override the context (profiling small cases)")
    ap.add_argument("--no-bar", action="store_true", help="skip timing the reference's Triton kernels")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    a.skip = {x for x in a.skip.split(",") if x} | ({"bar"} if a.no_bar else set())
    if a.impl == "reference":
        reference(a)
    else:
        ours(a)


if __name__ == "__main__":
    main()
