"""GPU: the W4A16 tree-verify step (csrc/verify_ops.cu + GEMM + attention) against an
fp32 torch restatement of the same Llama layer stack on the dequantised weights."""
import math

import numpy as np
import pytest
import torch

from oracle import tree_attn_oracle as orc

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qattention_b200 import _lib, quant
    from qattention_b200 import verify as vf


def _rmsnorm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _rope(x, pos, inv_freq):
    # x [..., T, D] rotate-half, positions [T]
    ang = pos.double()[:, None] * inv_freq.double()[None, :]
    cos, sin = torch.cat([ang.cos(), ang.cos()], -1).float(), torch.cat([ang.sin(), ang.sin()], -1).float()
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], -1)
    return x * cos + rot * sin


def _reference(model, tokens, cache0, L, b, d):
    c = model.cfg
    B, N = tokens.shape
    H, D, Hq, Hkv, F = c.hidden, c.head_dim, c.heads, c.kv_heads, c.ffn
    pos = (L + vf.tree_depths(b, d)).cuda()
    tree = torch.from_numpy(orc.ancestor_mask(N, b, d)).cuda()
    allowed = torch.cat([torch.ones(N, L, dtype=torch.bool, device="cuda"), tree], 1)   # [N, L+N]
    h = model.embed[tokens].float()                                                   # [B, N, H]
    for li, lw in enumerate(model.layers):
        deq = {k: quant.w4a16_dequantize(*lw[k]).float() for k in ("qkv", "o", "gate_up", "down")}
        x = _rmsnorm(h, lw["ln1"], c.rms_eps)
        qkv = (x @ deq["qkv"]).view(B, N, Hq + 2 * Hkv, D).permute(0, 2, 1, 3)
        q, k, v = qkv[:, :Hq], qkv[:, Hq:Hq + Hkv], qkv[:, Hq + Hkv:]
        q, k = _rope(q, pos, model.inv_freq), _rope(k, pos, model.inv_freq)
        kc, vc = cache0[li]
        K = torch.cat([kc[:, :, :L].float(), k], 2).repeat_interleave(Hq // Hkv, 1)
        V = torch.cat([vc[:, :, :L].float(), v], 2).repeat_interleave(Hq // Hkv, 1)
        s = (q @ K.transpose(-1, -2)) / math.sqrt(D)
        s = s.masked_fill(~allowed, float("-inf"))
        o = (torch.softmax(s, -1) @ V).permute(0, 2, 1, 3).reshape(B, N, Hq * D)
        h = h + o @ deq["o"]
        x = _rmsnorm(h, lw["ln2"], c.rms_eps)
        gu = x @ deq["gate_up"]
        act = torch.nn.functional.silu(gu[..., :F]) * gu[..., F:]
        h = h + act @ deq["down"]
    x = _rmsnorm(h, model.norm, c.rms_eps)
    return (x @ model.lm_head.float()).reshape(B * N, -1)


@pytest.mark.parametrize("b,d,L,B", [(2, 3, 128, 2), (4, 2, 200, 2), (2, 3, 128, 1)])
def test_verify_step_matches_fp32_model(b, d, L, B):
    # B=1: one sequence per GPU, as config 5 runs when its 8 sequences are sharded over 8 GPUs
    cfg = vf.LlamaConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000)
    model = vf.VerifyModel(cfg, "cuda", seed=3, std=0.05)
    N = (b ** (d + 1) - 1) // (b - 1)
    cache = model.new_cache(B, L, N, seed=4)
    cache0 = [(k.clone(), v.clone()) for k, v in cache]
    tokens = torch.randint(0, cfg.vocab, (B, N), generator=torch.Generator().manual_seed(5)).cuda()
    logits = model.step(tokens, cache, L, b, d).float()
    ref = _reference(model, tokens, cache0, L, b, d)
    err = (logits - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert torch.isfinite(logits).all()
    assert err <= 2e-2 * scale + 2e-2, f"max err {err:.3e}, max |logit| {scale:.3e}"
    assert _lib.device_error() == 0


def test_rope_writes_cache_and_rotates_q():
    M, n_per, Hq, Hkv, D = 6, 3, 2, 1, 64
    qkv = torch.randn(M, (Hq + 2 * Hkv) * D, device="cuda").half()
    orig = qkv.clone().float().view(M, Hq + 2 * Hkv, D)
    pos = torch.tensor([5, 6, 6, 9, 10, 10], dtype=torch.int32, device="cuda")
    inv = vf.llama31_inv_freq(vf.LlamaConfig(head_dim=D)).cuda()
    kc = torch.zeros(2, Hkv, 8, D, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    L = _lib.lib()
    _lib.check(L.qa_rope_qkv(qkv.data_ptr(), pos.data_ptr(), inv.data_ptr(), kc.data_ptr(), vc.data_ptr(), M, n_per,
                             Hq, Hkv, D, kc.stride(0), kc.stride(1), 4, torch.cuda.current_stream().cuda_stream),
               "qa_rope_qkv")
    torch.cuda.synchronize()
    q_ref = _rope(orig[:, :Hq].permute(1, 0, 2), pos, inv).permute(1, 0, 2)
    k_ref = _rope(orig[:, Hq:Hq + Hkv].permute(1, 0, 2), pos, inv).permute(1, 0, 2)
    assert (qkv.float().view(M, -1, D)[:, :Hq] - q_ref).abs().max() < 2e-2
    for m in range(M):
        bb, t = divmod(m, n_per)
        assert (kc[bb, :, 4 + t].float() - k_ref[m]).abs().max() < 2e-2
        assert torch.equal(vc[bb, :, 4 + t], qkv.view(M, -1, D)[m, Hq + Hkv:])
    assert kc[:, :, :4].abs().max() == 0 and kc[:, :, 7:].abs().max() == 0


def test_add_rmsnorm_and_silu_mul():
    M, Hd, F = 5, 512, 256
    h = torch.randn(M, Hd, device="cuda").half()
    dlt = torch.randn(M, Hd, device="cuda").half()
    w = torch.randn(Hd, device="cuda").half()
    out = torch.empty_like(h)
    h0 = h.clone()
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(L.qa_add_rmsnorm(h.data_ptr(), dlt.data_ptr(), w.data_ptr(), out.data_ptr(), M, Hd, 1e-5, st), "norm")
    gu = torch.randn(M, 2 * F, device="cuda").half()
    act = torch.empty(M, F, dtype=torch.float16, device="cuda")
    _lib.check(L.qa_silu_mul(gu.data_ptr(), act.data_ptr(), M, F, st), "silu")
    torch.cuda.synchronize()
    hs = h0.float() + dlt.float()
    assert (h.float() - hs).abs().max() < 1e-2
    ref = _rmsnorm(hs, w, 1e-5)
    assert (out.float() - ref).abs().max() < 2e-2 * ref.abs().max()
    a_ref = torch.nn.functional.silu(gu[:, :F].float()) * gu[:, F:].float()
    assert (act.float() - a_ref).abs().max() < 1e-2 * a_ref.abs().max() + 1e-3


def test_verify_step_cuda_graph_replay_matches_eager():
    # the whole verify step (every layer's GEMMs, attention and elementwise kernels
    # plus the LM head) captured once and replayed with new tokens
    cfg = vf.LlamaConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000)
    model = vf.VerifyModel(cfg, "cuda", seed=11, std=0.05)
    b, d, L, B = 2, 4, 96, 2
    N = (b ** (d + 1) - 1) // (b - 1)
    cache = model.new_cache(B, L, N, seed=12)
    tokens = torch.zeros(B, N, dtype=torch.int64, device="cuda")
    graph, logits = model.capture(tokens, cache, L, b, d)
    gen = torch.Generator().manual_seed(13)
    for _ in range(2):
        new = torch.randint(0, cfg.vocab, (B, N), generator=gen).cuda()
        tokens.copy_(new)
        graph.replay()
        torch.cuda.synchronize()
        eager = model.step(new, cache, L, b, d)
        assert torch.equal(logits, eager)
    assert _lib.device_error() == 0
