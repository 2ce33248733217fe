"""Attention oracle (test infrastructure only).

* :func:`sdpa_reference` -- the reference's own fallback path
  (``kairos/modules/dits/kairos_dit.py:269-276``): rearrange ``[B,S,N,D]`` to
  ``[B,N,S,D]`` and call ``F.scaled_dot_product_attention`` (non-causal, no
  mask, scale D^-1/2), here on CPU in fp32.
* :func:`fp8_attention_model` -- what the FP8 kernel computes, restated in
  torch: per-(batch, head) amax scaling of q and k to e4m3 (scale = amax/448),
  scores and softmax in fp32, then either P rounded to bf16 times the bf16 V
  (``bf16_pv``) or P rounded to e4m3 after scaling by 2^6 relative to the row
  max times V at its own per-head e4m3 scale; P V accumulated in fp32.
* :func:`quant_e4m3` optionally adds a second e4m3 term (the rounding
  residual); the models above do not use it, it measures what such a term buys.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

E4M3_MAX = 448.0


def sdpa_reference(q, k, v, num_heads):
    """q, k, v: [B, S, N*D] -> [B, S, N*D] float32 (CPU)."""
    B, S, HD = q.shape
    D = HD // num_heads
    f = lambda x: x.float().reshape(B, S, num_heads, D).transpose(1, 2)  # noqa: E731
    o = F.scaled_dot_product_attention(f(q), f(k), f(v))
    return o.transpose(1, 2).reshape(B, S, HD)


def sdpa_window_reference(q, k, v, num_heads, window_size):
    """Windowed attention (flash-attention window_size semantics, equal lengths):
    query i sees keys i - left .. i + right, -1 = unbounded; fp32 on CPU
    (the reference's flash_attention call with window_size, ``kairos_dit.py:232-277``,
    as SelfAttention issues it, ``:423-507``)."""
    B, S, HD = q.shape
    D = HD // num_heads
    left, right = window_size
    i = torch.arange(S)[:, None]
    j = torch.arange(S)[None, :]
    allow = torch.ones(S, S, dtype=torch.bool)
    if left >= 0:
        allow &= j >= i - left
    if right >= 0:
        allow &= j <= i + right
    f = lambda x: x.float().reshape(B, S, num_heads, D).transpose(1, 2)  # noqa: E731
    o = F.scaled_dot_product_attention(f(q), f(k), f(v), attn_mask=allow)
    return o.transpose(1, 2).reshape(B, S, HD)


def _e4m3(x):
    return x.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).float()


def quant_e4m3(x, num_heads, two_term=False):
    """Per-(batch, head) amax scaling; returns (dequantised x, scale [B,N]).

    With ``two_term`` the dequantised value is e4m3(x/s) + e4m3(x/s - e4m3(x/s)),
    both at scale s."""
    B, S, HD = x.shape
    D = HD // num_heads
    xh = x.float().reshape(B, S, num_heads, D)
    amax = xh.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    xs = xh / scale[:, None, :, None]
    hi = _e4m3(xs)
    if two_term:
        hi = hi + _e4m3(xs - hi)
    return (hi * scale[:, None, :, None]).reshape(B, S, HD), scale


def fp8_attention_model(q, k, v, num_heads, bf16_pv=True):
    B, S, HD = q.shape
    D = HD // num_heads
    qd, _ = quant_e4m3(q, num_heads)
    kd, _ = quant_e4m3(k, num_heads)
    f = lambda x: x.reshape(B, S, num_heads, D).transpose(1, 2)  # noqa: E731
    s = (f(qd) @ f(kd).transpose(-1, -2)) * D ** -0.5
    m = s.amax(-1, keepdim=True)
    p = torch.exp(s - m) * 64.0
    if bf16_pv:
        o = (p.bfloat16().float() @ f(v.bfloat16().float())) / p.sum(-1, keepdim=True)
    else:
        vd, _ = quant_e4m3(v, num_heads)
        o = (_e4m3(p) @ f(vd)) / p.sum(-1, keepdim=True)
    return o.transpose(1, 2).reshape(B, S, HD)
