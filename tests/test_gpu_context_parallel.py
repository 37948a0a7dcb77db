"""Context-parallel decode through the CUDA path, emulated on one GPU: the partial
results of every rank (paged_*_decode(..., context=(rank, world))) combined with
starkv_b200.context_parallel.combine_local must equal the single decode call
(tolerance 1e-2 abs + 1e-2 rel, inside the 2e-2 / 1e-2 bar against the reference).
Lengths include sequences with fewer 256-token tiles than ranks."""
import pytest
import torch

pytestmark = pytest.mark.gpu

LENS = [700, 129, 2048, 31, 5000, 256]


def _close(got, ref):
    got, ref = got.float(), ref.float()
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    assert torch.all(err <= 1e-2 + 1e-2 * ref.abs()), err.max().item()


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_bf16_context_split_combines_to_full_decode(world):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from starkv_b200.context_parallel import combine_local
    from starkv_b200.kernels.paged_decode import paged_starkv_decode
    from starkv_b200.workload import make_layer
    layer = make_layer(LENS, num_heads=8, seed=41, device=torch.device("cuda", 0))
    args = (layer.query, layer.kv_cache, layer.block_table, layer.seq_lens, layer.max_seq_len, layer.k_up,
            layer.k_ranks, layer.k_head_offsets, layer.k_width, layer.v_up_by_q, layer.cos_sin_cache, layer.scale)
    full = paged_starkv_decode(*args)
    parts = [tuple(t.clone() for t in paged_starkv_decode(*args, context=(r, world))) for r in range(world)]
    _close(combine_local(parts), full)


@pytest.mark.parametrize("world", [2, 4])
def test_quant_context_split_combines_to_full_decode(world):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from starkv_b200.context_parallel import combine_local
    from starkv_b200.kernels.paged_quant import paged_quant_decode
    from starkv_b200.workload import make_layer
    layer = make_layer(LENS, num_heads=8, quant=True, seed=42, device=torch.device("cuda", 0))
    args = (layer.query, layer.kv_cache, layer.block_table, layer.seq_lens, layer.max_seq_len, layer.row,
            layer.k_up, layer.head_of_lane, layer.k_tiles, layer.v_up_by_q, layer.cos_sin_cache, layer.scale)
    full = paged_quant_decode(*args)
    parts = [tuple(t.clone() for t in paged_quant_decode(*args, context=(r, world))) for r in range(world)]
    _close(combine_local(parts), full)
