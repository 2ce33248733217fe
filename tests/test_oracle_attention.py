"""CPU checks of the attention oracle (no GPU)."""
import torch
import torch.nn.functional as F

from oracle.attention import fp8_attention_model, quant_e4m3, sdpa_reference


def _cos(a, b):
    return F.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()


def test_sdpa_reference_matches_explicit_softmax():
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 50, 2 * 16, generator=g) for _ in range(3))
    o = sdpa_reference(q, k, v, 2)
    f = lambda x: x.reshape(1, 50, 2, 16).transpose(1, 2)  # noqa: E731
    ref = torch.softmax(f(q) @ f(k).transpose(-1, -2) / 4.0, -1) @ f(v)
    assert torch.allclose(o, ref.transpose(1, 2).reshape(1, 50, 32), atol=1e-5)


def test_quant_scale_is_per_head_amax():
    x = torch.zeros(1, 4, 2 * 8)
    x[0, 1, 3] = 896.0
    x[0, 2, 8 + 5] = -2.0
    xd, s = quant_e4m3(x, 2)
    assert torch.allclose(s, torch.tensor([[2.0, 2.0 / 448]]))
    assert xd[0, 1, 3] == 896.0 and xd[0, 2, 13] == -2.0


def test_bf16_pv_meets_cosine_contract_all_e4m3_does_not():
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 1024, 256, generator=g).bfloat16() for _ in range(3))
    ref = sdpa_reference(q, k, v, 2)
    assert _cos(fp8_attention_model(q, k, v, 2, bf16_pv=True), ref) >= 0.999
    assert _cos(fp8_attention_model(q, k, v, 2, bf16_pv=False), ref) < 0.999


def test_residual_term_is_the_e4m3_rounding_error():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1, 64, 2 * 128, generator=g)
    one, s = quant_e4m3(x, 2)
    two, _ = quant_e4m3(x, 2, two_term=True)
    assert (two - x).abs().max() < (one - x).abs().max() / 4


def test_window_reference_unbounded_is_full_attention():
    from oracle.attention import sdpa_window_reference
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 40, 32, generator=g) for _ in range(3))
    assert torch.allclose(sdpa_window_reference(q, k, v, 2, (-1, -1)), sdpa_reference(q, k, v, 2), atol=1e-6)
    # a zero-width window is the identity on v
    assert torch.allclose(sdpa_window_reference(q, k, v, 2, (0, 0)), v, atol=1e-6)
