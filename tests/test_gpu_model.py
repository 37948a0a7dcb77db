"""GPU check of a whole (small) STAR-KV Llama decode step (starkv_b200.model):
decoding a few tokens one step at a time from empty paged caches gives the same
last-position logits as a dense fp32 recomputation of the sequences with causal
attention (compressed layers: K lifted per head from the codes and rotated, V
lifted; full-rank layers: stock attention). bf16 activations and caches on the GPU,
so the bound is relative: ||logits - ref|| <= 3% ||ref||.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

STEPS, BATCH = 24, 3


def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def small_config():
    from starkv_b200.model import ModelConfig
    return ModelConfig(hidden=512, heads=4, ffn=1024, vocab=512, layers=3, full_layers=(0,), max_pos=256, seed=5)


def dense_reference(model, tokens):
    """fp32 forward of whole sequences tokens [B, T] -> logits of the last position."""
    from starkv_b200.layer import rope
    from starkv_b200.model import rms_norm
    cfg = model.cfg
    B, T = tokens.shape
    pos = torch.arange(T, device=tokens.device)
    x = model.embed[tokens].float()
    cs = model.cos_sin_cache
    mask = torch.ones(T, T, dtype=torch.bool, device=tokens.device).tril()

    def attend(q, k, v):   # [B, T, H, 128] each
        s = torch.einsum("bthd,bshd->bhts", q, k) * 128 ** -0.5
        s = s.masked_fill(~mask, float("-inf"))
        return torch.einsum("bhts,bshd->bthd", s.softmax(-1), v)

    for ly in model.layers:
        a = ly["attn"]
        h = rms_norm(x, ly["norms"][0].float(), cfg.rms_eps)
        if ly["full"]:
            H = a.heads
            q, k, v = F.linear(h, a.wqkv.float()).view(B, T, 3, H, 128).unbind(2)
            q = rope(q.reshape(B * T, H, 128), pos.repeat(B), cs).view(B, T, H, 128)
            k = rope(k.reshape(B * T, H, 128), pos.repeat(B), cs).view(B, T, H, 128)
            o = attend(q, k, v)
        else:
            H = a.num_heads
            q = rope(F.linear(h, a.wq.float()).view(B * T, H, 128), pos.repeat(B), cs).view(B, T, H, 128)
            codes = F.linear(h, a.kv_down.float())
            kc, vc = codes[..., :a.k_width], codes[..., a.k_width:]
            ks = []
            for hh, (r, o) in enumerate(zip(a.k_ranks_host, a.k_head_offsets.tolist())):
                ks.append(kc[..., o:o + r] @ a.k_up[o:o + r].float())
            k = rope(torch.stack(ks, 2).reshape(B * T, H, 128), pos.repeat(B), cs).view(B, T, H, 128)
            v = torch.einsum("btr,hrd->bthd", vc, a.v_up_by_q.float())
            o = attend(q, k, v)
        x = x + F.linear(o.reshape(B, T, -1), (a.wo).float())
        h = rms_norm(x, ly["norms"][1].float(), cfg.rms_eps)
        g, u = F.linear(h, ly["gate_up"].float()).chunk(2, dim=-1)
        x = x + F.linear(F.silu(g) * u, ly["down"].float())
    return F.linear(rms_norm(x, model.final_norm.float(), cfg.rms_eps), model.lm_head.float())[:, -1]


def test_model_decode_matches_dense_reference():
    from starkv_b200.model import StarKVModel
    dev = cuda()
    model = StarKVModel(small_config(), dev)
    g = torch.Generator(device=dev).manual_seed(1)
    tokens = torch.randint(0, model.cfg.vocab, (BATCH, STEPS), generator=g, device=dev)
    pages = -(-STEPS // 16)
    caches = model.allocate_caches(BATCH * pages + 1)
    bt = (torch.arange(BATCH * pages, device=dev, dtype=torch.int32).view(BATCH, pages) + 1)
    for t in range(STEPS):
        pos = torch.full((BATCH,), t, device=dev)
        slots = bt[:, t // 16].long() * 16 + t % 16
        seq_lens = torch.full((BATCH,), t + 1, dtype=torch.int32, device=dev)
        logits = model.decode_step(tokens[:, t], pos, caches, bt, seq_lens, STEPS, slots)
    ref = dense_reference(model, tokens)
    rel = (logits - ref).norm() / ref.norm()
    assert float(rel) < 3e-2, f"relative error {float(rel):.3e}"
    agree = (logits.argmax(-1) == ref.argmax(-1)).float().mean()
    assert float(agree) >= 2 / 3


def test_model_from_fused_checkpoint_file(tmp_path):
    """The model served from a fused_weights.pt written in the reference layout
    (random-init factors, one layer left out and so full-rank): the loader's layout
    reaches the kernels, and decoding matches the dense recomputation."""
    from starkv_b200.checkpoint import write_synthetic_checkpoint
    from starkv_b200.model import StarKVModel, checkpoint_layer_ranks
    dev = cuda()
    cfg = small_config()
    path = tmp_path / "fused_weights.pt"
    write_synthetic_checkpoint(str(path), checkpoint_layer_ranks(cfg), cfg.hidden, cfg.heads, seed=2)
    model = StarKVModel(small_config(), dev, checkpoint=str(path))
    assert [ly["full"] for ly in model.layers] == [True, False, False]
    g = torch.Generator(device=dev).manual_seed(3)
    tokens = torch.randint(0, model.cfg.vocab, (BATCH, STEPS), generator=g, device=dev)
    pages = -(-STEPS // 16)
    caches = model.allocate_caches(BATCH * pages + 1)
    bt = (torch.arange(BATCH * pages, device=dev, dtype=torch.int32).view(BATCH, pages) + 1)
    for t in range(STEPS):
        pos = torch.full((BATCH,), t, device=dev)
        slots = bt[:, t // 16].long() * 16 + t % 16
        seq_lens = torch.full((BATCH,), t + 1, dtype=torch.int32, device=dev)
        logits = model.decode_step(tokens[:, t], pos, caches, bt, seq_lens, STEPS, slots)
    ref = dense_reference(model, tokens)
    rel = (logits - ref).norm() / ref.norm()
    assert float(rel) < 3e-2, f"relative error {float(rel):.3e}"
