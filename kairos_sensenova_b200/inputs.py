"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (there is no dataset on this path).

GDN (configs 0/1): q, k, v ~ N(0,1) drawn in that order, beta = sigmoid(N(0,1)),
g = -softplus(N(0,1)); q/k are L2-normalised by the op
(``use_qk_l2norm_in_kernel=True``).  Attention (config 2): q, k, v ~ N(0,1) bf16.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def gdn_inputs(B, T, H, K, V, seed=0, device='cuda', dtype=torch.bfloat16):
    gen = _gen(device, seed)
    q = torch.randn(B, T, H, K, generator=gen, device=device).to(dtype)
    k = torch.randn(B, T, H, K, generator=gen, device=device).to(dtype)
    v = torch.randn(B, T, H, V, generator=gen, device=device).to(dtype)
    beta = torch.randn(B, T, H, generator=gen, device=device).sigmoid().to(dtype)
    g = -F.softplus(torch.randn(B, T, H, generator=gen, device=device))
    return q, k, v, g, beta


def attn_inputs(B, S, H, D, seed=1, device='cuda', dtype=torch.bfloat16):
    gen = _gen(device, seed)
    q = torch.randn(B, S, H * D, generator=gen, device=device).to(dtype)
    k = torch.randn(B, S, H * D, generator=gen, device=device).to(dtype)
    v = torch.randn(B, S, H * D, generator=gen, device=device).to(dtype)
    return q, k, v
