"""CPU restatement of the benchmark's hybrid block (test infrastructure only):
GatedDeltaNet chain then attention chain, single process (the Ulysses
re-partition is a permutation and does not change the result).

The GDN chain follows ``GatedDeltaNet.forward`` (``fla/layers/gated_deltanet.py:234-315``);
the attention chain is q/k/v projections, softmax attention (the reference's
SDPA fallback, ``kairos_dit.py:269-276``) and the output projection.
"""
from __future__ import annotations

import torch

from .attention import sdpa_reference
from .gdn import gdn_chunk
from .layers import gates, rmsnorm_gated, rmsnorm_rope, short_conv_silu


def gdn_chain(w, x, H, D, eps=1e-5, heads=None):
    """x [T, hidden] fp32; w: dict of CPU fp32 weights ([out, in] like nn.Linear).
    ``heads`` restricts the mixer to a subset of heads (used for bounded CPU
    samples); the returned output then covers those heads' contribution only."""
    T = x.shape[0]
    hs = list(range(H)) if heads is None else list(heads)
    cols = torch.cat([torch.arange(h * D, (h + 1) * D) for h in hs])
    q = short_conv_silu((x @ w['Wq'][cols].t())[None], w['cq'][cols])
    k = short_conv_silu((x @ w['Wk'][cols].t())[None], w['ck'][cols])
    v = short_conv_silu((x @ w['Wv'][cols].t())[None], w['cv'][cols])
    g, beta = gates(x @ w['Wa'][hs].t(), x @ w['Wb'][hs].t(), w['A_log'][hs], w['dt_bias'][hs])
    n = len(hs)
    o, _ = gdn_chunk(q.reshape(1, T, n, D), k.reshape(1, T, n, D), v.reshape(1, T, n, D),
                     g[None], beta[None], None, None, False, use_qk_l2norm=True)
    gate = (x @ w['Wg'][cols].t()).reshape(T, n, D)
    y = rmsnorm_gated(o[0], gate, w['o_norm_w'], eps).reshape(T, n * D)
    return y @ w['Wo'][:, cols].t()


def freqs_cis_3d(D, f, h, w, theta=10000.0):
    """Per-token complex RoPE factors (``kairos_dit.py:312-322,1217-1221``)."""
    def one(dim, end):
        fr = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].double() / dim))
        ang = torch.outer(torch.arange(end, dtype=torch.float64), fr)
        return torch.polar(torch.ones_like(ang), ang)
    a, b, c = one(D - 2 * (D // 3), f), one(D // 3, h), one(D // 3, w)
    return torch.cat([a.view(f, 1, 1, -1).expand(f, h, w, -1), b.view(1, h, 1, -1).expand(f, h, w, -1),
                      c.view(1, 1, w, -1).expand(f, h, w, -1)], -1).reshape(f * h * w, -1)


def attn_chain(w, x, H, D, heads=None, freqs=None, eps=1e-6, work_share=False):
    """q/k projections with full-dim RMSNorm + RoPE (``SelfAttention.forward``,
    ``kairos_dit.py:452-456``), SDPA, output projection.  With ``heads`` only
    those heads' attention is computed and the norm still spans all heads;
    ``work_share=True`` (CPU timing samples only) projects just those heads and
    normalises over their channels, so the sample does exactly their share of
    the work."""
    T = x.shape[0]
    hs = list(range(H)) if heads is None else list(heads)
    cols = torch.cat([torch.arange(h * D, (h + 1) * D) for h in hs])
    if freqs is None:
        freqs = freqs_cis_3d(D, T, 1, 1)
    nq, nk = w.get('nq', torch.ones(H * D)), w.get('nk', torch.ones(H * D))
    if work_share:
        q = rmsnorm_rope((x @ w['Aq'][cols].t())[None], nq[cols], freqs, len(hs), eps).float()
        k = rmsnorm_rope((x @ w['Ak'][cols].t())[None], nk[cols], freqs, len(hs), eps).float()
    else:
        q = rmsnorm_rope((x @ w['Aq'].t())[None], nq, freqs, H, eps).float()[..., cols]
        k = rmsnorm_rope((x @ w['Ak'].t())[None], nk, freqs, H, eps).float()[..., cols]
    v = (x @ w['Av'][cols].t())[None]
    o = sdpa_reference(q, k, v, len(hs))[0]
    return o @ w['Ao'][:, cols].t()


def hybrid_forward(w, x, H, D, eps=1e-5):
    return attn_chain(w, gdn_chain(w, x, H, D, eps), H, D)


def weights_of(block):
    """CPU fp32 copies of a kairos_sensenova_b200.hybrid.HybridBlock's weights."""
    names = ('Wq', 'Wk', 'Wv', 'Wg', 'Wa', 'Wb', 'Wo', 'Aq', 'Ak', 'Av', 'Ao', 'cq', 'ck', 'cv',
             'A_log', 'dt_bias', 'o_norm_w', 'nq', 'nk')
    return {n: getattr(block, n).detach().float().cpu() for n in names}
