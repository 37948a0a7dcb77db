"""GPU parity of the prefill attention kernel (starkv_prefill_attention, the library's
replacement for the reference prefill's flash_attn_varlen_func, attention.py:246-250)
against a float32 torch restatement: per prompt, softmax(scale q k^T) v over keys
<= query.

Tolerance: bf16 / f16 inputs, f32 accumulation, P rounded to the input type before
P.V (as flash attention does): |out - ref| <= 2e-2 + 2e-2 |ref| element-wise for
bf16, 5e-3 + 5e-3 |ref| for f16.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def reference(q, k, v, lens, scale):
    T, H, _ = q.shape
    Gk, Gv = H // k.shape[1], H // v.shape[1]
    out = torch.empty(T, H, 128, dtype=torch.float32, device=q.device)
    s0 = 0
    for L in lens:
        qs = q[s0:s0 + L].float().transpose(0, 1)
        ks = k[s0:s0 + L].float().transpose(0, 1).repeat_interleave(Gk, dim=0)
        vs = v[s0:s0 + L].float().transpose(0, 1).repeat_interleave(Gv, dim=0)
        s = scale * qs @ ks.transpose(1, 2)
        mask = torch.ones(L, L, dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
        out[s0:s0 + L] = (torch.softmax(s, dim=-1) @ vs).transpose(0, 1)
        s0 += L
    return out


def run_case(lens, H, Hk, Hv, dtype, seed=0, mag=1.0):
    from starkv_b200.kernels.prefill import prefill_attention
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(seed)
    T = sum(lens)
    q = (mag * torch.randn(T, H, 128, generator=g, device=dev)).to(dtype)
    k = (mag * torch.randn(T, Hk, 128, generator=g, device=dev)).to(dtype)
    v = torch.randn(T, Hv, 128, generator=g, device=dev).to(dtype)
    scale = 128 ** -0.5
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out = prefill_attention(q, k, v, lens, scale, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = reference(q, k, v, lens, scale)
    tol = 2e-2 if dtype == torch.bfloat16 else 5e-3
    err = (out.float() - ref).abs()
    assert torch.isfinite(out.float()).all()
    assert (err <= tol + tol * ref.abs()).all(), float(err.max())
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_mha_ragged_prompts(dtype):
    # lengths around the 128-token tile: 1, partial, exact, one over, several tiles
    run_case([1, 5, 127, 128, 129, 300], H=4, Hk=4, Hv=4, dtype=dtype)


def test_prefill_gqa_v_per_query_head():
    # the layer's layout: K per KV head (4 query heads each), V per query head
    run_case([200, 77, 513], H=8, Hk=2, Hv=8, dtype=torch.bfloat16, seed=1)


def test_prefill_gqa_v_per_kv_head():
    # the reference's layout: K and V per KV head
    run_case([256, 31], H=8, Hk=4, Hv=4, dtype=torch.bfloat16, seed=2)


def test_prefill_long_prompt_large_logits():
    # 9 key tiles for the last query tile; logits large enough that the running
    # max changes from tile to tile (output rescaling)
    run_case([1100], H=2, Hk=1, Hv=2, dtype=torch.bfloat16, seed=3, mag=3.0)


def test_prefill_strided_inputs_and_empty():
    from starkv_b200.kernels.prefill import prefill_attention
    dev = cuda()
    g = torch.Generator(device=dev).manual_seed(4)
    lens = [70, 190]
    T, H = sum(lens), 4
    # q, k, v as head slices of one packed [T, 3H, 128] tensor (token stride 3H*128)
    qkv = torch.randn(T, 3 * H, 128, generator=g, device=dev).to(torch.bfloat16)
    q, k, v = qkv[:, :H], qkv[:, H:2 * H], qkv[:, 2 * H:]
    out = prefill_attention(q, k, v, lens, 0.1)
    ref = reference(q, k, v, lens, 0.1)
    assert ((out.float() - ref).abs() <= 2e-2 + 2e-2 * ref.abs()).all()
    empty = prefill_attention(q[:0], k[:0], v[:0], [], 0.1)
    assert empty.shape == (0, H, 128)


def test_prefill_repeatable():
    a = run_case([300, 45], H=4, Hk=2, Hv=4, dtype=torch.bfloat16, seed=5)
    b = run_case([300, 45], H=4, Hk=2, Hv=4, dtype=torch.bfloat16, seed=5)
    assert torch.equal(a, b)
