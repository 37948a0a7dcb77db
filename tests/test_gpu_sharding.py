"""Head sharding through the CUDA path on one GPU: a layer's inputs are split by
KV head with the host logic of starkv_b200.sharding (each shard: its heads' K
codes and k_up rows, its query and v_up_by_q rows, the whole V latent), each
shard is decoded by paged_starkv_decode, and every head's output must match the
unsharded call (same kernels, different lane packing; tolerance 1e-2 abs +
1e-2 rel, inside the 2e-2 / 1e-2 bar against the reference)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_decode_matches_unsharded(world):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from starkv_b200.kernels.paged_decode import paged_starkv_decode
    from starkv_b200.sharding import lpt_shard, query_heads, shard_lanes
    from starkv_b200.workload import make_layer
    dev = torch.device("cuda", 0)
    layer = make_layer([700, 129, 2048, 31], num_heads=8, seed=31, device=dev)
    W = layer.k_width

    def run(q, cache, k_up, ranks, offs, width, v_up):
        return paged_starkv_decode(q, cache, layer.block_table, layer.seq_lens, layer.max_seq_len, k_up,
                                   torch.tensor(ranks, dtype=torch.int32, device=dev),
                                   torch.tensor(offs, dtype=torch.int32, device=dev), width, v_up,
                                   layer.cos_sin_cache, layer.scale)

    full = run(layer.query, layer.kv_cache, layer.k_up, layer.ranks, layer.offsets, W, layer.v_up_by_q).float()
    for heads in lpt_shard(layer.ranks, world):
        lr, lo, lw, lanes = shard_lanes(layer.ranks, heads)
        qh = query_heads(heads, 1)
        idx = torch.tensor(lanes, device=dev)
        cache = torch.cat([layer.kv_cache.index_select(2, idx), layer.kv_cache[:, :, W:]], 2).contiguous()
        out = run(layer.query[:, qh].contiguous(), cache, layer.k_up.index_select(0, idx).contiguous(), lr, lo, lw,
                  layer.v_up_by_q[qh].contiguous()).float()
        ref = full[:, qh]
        assert torch.all((out - ref).abs() <= 1e-2 + 1e-2 * ref.abs()), (out - ref).abs().max().item()
