"""GPU parity of the FP8 (e4m3, per-head amax) attention kernel.

Contract: cosine similarity >= 0.999 against the reference's bf16
``F.scaled_dot_product_attention`` path (``kairos_dit.py:269-276``); small
cases are also checked against the fp32 CPU oracle and the FP8 model."""
import pytest
import torch
import torch.nn.functional as F

from oracle.attention import fp8_attention_model, sdpa_reference

pytestmark = pytest.mark.gpu
COS = 0.999


def cos(a, b):
    return F.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0).item()


@pytest.mark.parametrize('B,S,H', [(1, 1, 2), (1, 100, 2), (2, 257, 3), (1, 1000, 4)])
def test_attn_fp8_small_vs_oracle(B, S, H):
    from kairos_sensenova_b200.attention import AttentionModule
    gen = torch.Generator().manual_seed(S)
    q, k, v = (torch.randn(B, S, H * 128, generator=gen).bfloat16() for _ in range(3))
    o = AttentionModule(H)(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    assert o.shape == q.shape and o.dtype == torch.bfloat16
    ref = sdpa_reference(q, k, v, H)
    model = fp8_attention_model(q, k, v, H)
    assert cos(o.cpu(), ref) >= COS
    # the kernel is close to the FP8 model (same quantisation points)
    assert (o.cpu().float() - model).abs().max().item() < 2e-2 * model.abs().max().item() + 1e-2


def test_attn_fp8_config2_full_size_vs_bf16_sdpa():
    """B=1, H=24, T=32760, d=128, q,k,v ~ N(0,1) bf16 seed 1."""
    from kairos_sensenova_b200.attention import AttentionModule
    from kairos_sensenova_b200.inputs import attn_inputs
    H = 24
    q, k, v = attn_inputs(1, 32760, H, 128, seed=1)
    o = AttentionModule(H)(q, k, v)
    f = lambda x: x.reshape(1, 32760, H, 128).transpose(1, 2)  # noqa: E731
    ref = F.scaled_dot_product_attention(f(q), f(k), f(v)).transpose(1, 2).reshape(1, 32760, H * 128)
    c = cos(o, ref)
    print(f'config2 cosine vs bf16 SDPA: {c:.6f}')
    assert c >= COS
    for h in range(H):
        sl = slice(h * 128, (h + 1) * 128)
        assert cos(o[..., sl], ref[..., sl]) >= COS


def test_attn_fp8_structured_inputs():
    """Peaked attention (large logits) and per-head scale differences."""
    from kairos_sensenova_b200.attention import AttentionModule
    gen = torch.Generator().manual_seed(9)
    B, S, H = 1, 512, 2
    q = torch.randn(B, S, H * 128, generator=gen)
    k = q + 0.1 * torch.randn(B, S, H * 128, generator=gen)   # near-diagonal attention
    q[..., :128] *= 4.0                                       # head 0 much sharper
    v = torch.randn(B, S, H * 128, generator=gen) * 3.0
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    o = AttentionModule(H)(q.cuda(), k.cuda(), v.cuda())
    assert cos(o.cpu(), sdpa_reference(q, k, v, H)) >= COS


def test_attn_module_errors():
    from kairos_sensenova_b200.attention import AttentionModule
    x = torch.zeros(1, 8, 256, device='cuda', dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        AttentionModule(2)(x, x, x, attn_mask=torch.ones(8, 8, device='cuda'))
    with pytest.raises(ValueError):
        AttentionModule(4)(x, x, x)     # D = 64 unsupported


def test_attn_fp8_strided_qkv_views_match_contiguous():
    """q/k/v as column slices of one fused projection are read in place."""
    from kairos_sensenova_b200.attention import attention_fp8
    gen = torch.Generator().manual_seed(31)
    S, H = 700, 2
    fused = torch.randn(1, S, 3 * H * 128 + 8, generator=gen).bfloat16().cuda()
    q, k, v = (fused[..., i * H * 128:(i + 1) * H * 128] for i in range(3))
    o1 = attention_fp8(q, k, v, H)
    o2 = attention_fp8(q.contiguous(), k.contiguous(), v.contiguous(), H)
    assert torch.equal(o1, o2)


@pytest.mark.parametrize('S,H,window', [(1000, 2, (64, 64)), (777, 3, (0, 300)), (4096, 2, (300, 10)),
                                        (2000, 2, (-1, 5)), (3000, 2, (100, -1)), (300, 2, (3, 3))])
def test_attn_fp8_sliding_window_vs_oracle(S, H, window):
    """flash-attention window_size semantics: query i attends keys i - left .. i + right
    (the reference's SelfAttention, kairos_dit.py:423-507, calls attention that way)."""
    from kairos_sensenova_b200.attention import AttentionModule
    from oracle.attention import sdpa_window_reference
    gen = torch.Generator().manual_seed(S + 7)
    q, k, v = (torch.randn(1, S, H * 128, generator=gen).bfloat16() for _ in range(3))
    o = AttentionModule(H)(q.cuda(), k.cuda(), v.cuda(), window_size=window)
    torch.cuda.synchronize()
    ref = sdpa_window_reference(q, k, v, H, window)
    assert torch.isfinite(o.float()).all()
    assert cos(o.cpu(), ref) >= COS
    # the window changes the result (it is not ignored)
    if window != (-1, -1) and min(window) >= 0:
        assert cos(o.cpu(), sdpa_reference(q, k, v, H)) < 0.99


def test_attn_fp8_dilated_window_like_reference_self_attention():
    """SelfAttention with dilated_length d > 1 rearranges b (n d l) c -> (b d) (n l) c before
    a windowed call with window (L*w, L*w) (kairos_dit.py:452-495); the same here."""
    from einops import rearrange
    from kairos_sensenova_b200.attention import AttentionModule
    from oracle.attention import sdpa_window_reference
    H, d, L, w, n = 2, 2, 16, 3, 40
    gen = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(1, n * d * L, H * 128, generator=gen).bfloat16() for _ in range(3))
    r = lambda x: rearrange(x, 'b (n d l) c -> (b d) (n l) c', l=L, d=d)  # noqa: E731
    qd, kd, vd = r(q), r(k), r(v)
    o = AttentionModule(H)(qd.cuda(), kd.cuda(), vd.cuda(), window_size=(L * w, L * w))
    ref = sdpa_window_reference(qd, kd, vd, H, (L * w, L * w))
    assert cos(o.cpu(), ref) >= COS
