"""CPU restatement of the GatedDeltaNet layer math around the chunk op and of
the Ulysses re-partition (test infrastructure only).

* :func:`short_conv_silu` -- ``ShortConvolution`` forward, causal depthwise
  conv + SiLU (``fla/modules/convolution.py:53-140``; weight ``[C, W]``).
* :func:`gates` -- ``beta = sigmoid(b)``, ``g = -exp(A_log) softplus(a + dt_bias)``
  (``fla/layers/gated_deltanet.py:267-271``).
* :func:`rmsnorm_gated` -- ``FusedRMSNormGated`` with swish gate
  (``fla/modules/fused_norm_gate.py:60-110``).
* :func:`gated_deltanet_forward` -- ``GatedDeltaNet.forward`` (``gated_deltanet.py:202-319``)
  in chunk mode with the weights of a state dict.
* :func:`seq_to_head_expected` / :func:`head_to_seq_expected` -- what each
  rank must hold after the Ulysses all-to-all (``kairos/modules/utils/tp_utils.py:84-254``),
  as slicing of the full tensor.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .gdn import gdn_chunk


def short_conv_silu(x, w, bias=None):
    """x [B,T,C], w [C,W] -> SiLU(causal conv), computed in fp32."""
    B, T, C = x.shape
    W = w.shape[1]
    xp = F.pad(x.float().transpose(1, 2), (W - 1, 0))
    y = F.conv1d(xp, w.float()[:, None, :], bias=None if bias is None else bias.float(), groups=C)
    return F.silu(y).transpose(1, 2)


def gates(a, b, A_log, dt_bias, allow_neg_eigval=False):
    beta = b.float().sigmoid()
    if allow_neg_eigval:
        beta = beta * 2.0
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, beta


def rmsnorm_gated(x, gate, weight, eps):
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    gf = gate.float()
    return xf * rstd * weight.float() * gf * torch.sigmoid(gf)


def gated_deltanet_forward(sd, x, num_heads, head_k_dim, head_v_dim, norm_eps=1e-5, emulate_bf16=True):
    """Chunk-mode forward of GatedDeltaNet from a state dict (fp32 CPU math,
    bf16 rounding at the layer's activation boundaries when ``emulate_bf16``)."""
    r = (lambda t: t.bfloat16().float()) if emulate_bf16 else (lambda t: t)
    B, T, _ = x.shape
    xf = x.float()
    lin = lambda name: r(xf @ sd[f'{name}.weight'].float().t())  # noqa: E731
    q = r(short_conv_silu(lin('q_proj'), sd['q_conv1d.weight'][:, 0]))
    k = r(short_conv_silu(lin('k_proj'), sd['k_conv1d.weight'][:, 0]))
    v = r(short_conv_silu(lin('v_proj'), sd['v_conv1d.weight'][:, 0]))
    g, beta = gates(lin('a_proj'), lin('b_proj'), sd['A_log'], sd['dt_bias'])
    beta = r(beta)
    q = q.reshape(B, T, num_heads, head_k_dim)
    k = k.reshape(B, T, num_heads, head_k_dim)
    v = v.reshape(B, T, num_heads, head_v_dim)
    o, _ = gdn_chunk(q, k, v, g, beta, None, None, False, use_qk_l2norm=True, emulate_bf16=emulate_bf16)
    gate = lin('g_proj').reshape(B, T, num_heads, head_v_dim)
    o = r(rmsnorm_gated(r(o), gate, sd['o_norm.weight'], norm_eps)).reshape(B, T, -1)
    return o @ sd['o_proj.weight'].float().t()


def seq_to_head_expected(full, rank, world, dims=None):
    """full [B, N, D] -> rank's [B, N, D_local] after all2all_seq_to_head."""
    D = full.shape[-1]
    dims = dims or [D // world] * world
    off = sum(dims[:rank])
    return full[:, :, off:off + dims[rank]]


def head_to_seq_expected(full, rank, world):
    """full [B, N, D] -> rank's [B, N/P, D] after all2all_head_to_seq."""
    n = full.shape[1] // world
    return full[:, rank * n:(rank + 1) * n]


def rmsnorm_rope(x, weight, freqs, num_heads, eps=1e-6):
    """``rope_apply(norm(x))`` as the reference computes it: apex FusedRMSNorm
    over the full dim in fp32 -> bf16, then (``kairos_dit.py:324-329``) fp16
    complex pairs times the (double) complex factors, result cast to bf16.
    x: [B, S, N*D]; freqs: complex [S, D/2]."""
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()).bfloat16()
    B, S, HD = y.shape
    c = torch.view_as_complex(y.reshape(B, S, num_heads, -1, 2).to(torch.float16).float().contiguous())
    out = torch.view_as_real(c.to(torch.complex128) * freqs.reshape(1, S, 1, -1)).flatten(3)
    return out.reshape(B, S, HD).bfloat16()
