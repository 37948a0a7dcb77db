"""GPU parity of the fused K/V down-projection + cache write (starkv_kv_down_cache_write:
model.py:70 codes = F.linear(hidden, kv_down), then the cache write of
attention.py:179-185) against torch: the same GEMM in float32, rounded once to the
cache dtype, at the same slots.

Tolerance: each written element within one unit in the last place of the cache dtype
of the float32 result plus 2^-11 of the dot product's sum of |x w| (the tensor cores'
accumulation is not an exact float32 sum, and the split-K adds in another order);
the reference computation itself, F.linear on cuBLAS, is checked against the same
bound. Rows the step does not own stay untouched bit for bit.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def ulp(x: torch.Tensor, dtype) -> torch.Tensor:
    mant = 7 if dtype == torch.bfloat16 else 10
    e = torch.floor(torch.log2(x.abs().clamp(min=2.0 ** -14)))
    return 2.0 ** (e - mant)


def run(n, hidden, width, dtype, slot_dtype=torch.int32, pad=0, seed=0):
    from starkv_b200.kernels.paged_decode import kv_down_write
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(seed)
    x = (torch.randn(n, hidden, generator=g, device=dev) / 8).to(dtype)
    w = (torch.randn(width, hidden, generator=g, device=dev) / 8).to(dtype)
    num_blocks, bs = 64, 16
    cache = torch.randn(num_blocks, bs, width + pad, generator=g, device=dev).to(dtype)
    before = cache.clone()
    slots = torch.randperm(num_blocks * bs - bs, generator=g, device=dev)[:n] + bs   # block 0 is the null block
    slots = slots.to(slot_dtype)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    kv_down_write(x, w, cache, slots, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = x.float() @ w.float().t()
    tol = ulp(ref, dtype) + 2.0 ** -11 * (x.float().abs() @ w.float().abs().t())
    got = cache.view(-1, width + pad)[slots.long(), :width].float()
    assert ((got - ref).abs() <= tol).all(), float(((got - ref).abs() / tol).max())
    lib_ref = torch.nn.functional.linear(x, w).float()     # what the reference computes (model.py:70)
    assert ((lib_ref - ref).abs() <= tol).all()
    # everything else untouched: other rows, and the row tail past the codes
    mask = torch.ones(num_blocks * bs, dtype=torch.bool, device=dev)
    mask[slots.long()] = False
    assert torch.equal(cache.view(-1, width + pad)[mask], before.view(-1, width + pad)[mask])
    if pad:
        assert torch.equal(cache.view(-1, width + pad)[slots.long(), width:], before.view(-1, width + pad)[slots.long(), width:])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_kv_down_write_config_geometry(dtype):
    # Llama-2-7B hidden, config-2 code width (W 1392 + rv 1536), a decode batch of 64
    run(64, 4096, 2928, dtype)


def test_kv_down_write_ragged_sizes():
    # a token count that is not a multiple of 16, a width ending inside a 128-channel
    # tile and inside an 8-channel group, int64 slots, padded cache rows
    run(37, 1024, 200, torch.bfloat16, slot_dtype=torch.int64, pad=24, seed=1)
    run(1, 512, 8, torch.bfloat16, seed=2)


def test_kv_down_write_many_tokens():
    # more tokens than one 256-token launch column (a prefill chunk)
    run(300, 2048, 2928, torch.bfloat16, seed=3)


def test_kv_down_write_padding_rows_go_to_the_null_block():
    from starkv_b200.kernels.paged_decode import kv_down_write
    dev = cuda()
    x = torch.randn(4, 512, device=dev).to(torch.bfloat16)
    w = torch.randn(96, 512, device=dev).to(torch.bfloat16)
    cache = torch.zeros(8, 16, 96, device=dev).to(torch.bfloat16)
    slots = torch.tensor([17, -1, 33, 50], dtype=torch.int32, device=dev)
    kv_down_write(x, w, cache, slots)
    ref = x.float() @ w.float().t()
    tol = ulp(ref, torch.bfloat16) + 2.0 ** -11 * (x.float().abs() @ w.float().abs().t())
    flat = cache.view(-1, 96).float()
    for row, s in ((0, 17), (2, 33), (3, 50)):
        assert ((flat[s] - ref[row]).abs() <= tol[row]).all()
    assert ((flat[0] - ref[1]).abs() <= tol[1]).all()   # slot -1 -> slot 0, the reserved null block
    written = torch.zeros(flat.shape[0], dtype=torch.bool, device=dev)
    written[[0, 17, 33, 50]] = True
    assert int(flat[~written].abs().sum()) == 0          # no other row touched
