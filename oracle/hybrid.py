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
from .layers import gates, rmsnorm_gated, short_conv_silu


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


def attn_chain(w, x, H, D, heads=None):
    T = x.shape[0]
    hs = list(range(H)) if heads is None else list(heads)
    cols = torch.cat([torch.arange(h * D, (h + 1) * D) for h in hs])
    q, k, v = ((x @ w[n][cols].t())[None] for n in ('Aq', 'Ak', 'Av'))
    o = sdpa_reference(q, k, v, len(hs))[0]
    return o @ w['Ao'][:, cols].t()


def hybrid_forward(w, x, H, D, eps=1e-5):
    return attn_chain(w, gdn_chain(w, x, H, D, eps), H, D)


def weights_of(block):
    """CPU fp32 copies of a kairos_sensenova_b200.hybrid.HybridBlock's weights."""
    names = ('Wq', 'Wk', 'Wv', 'Wg', 'Wa', 'Wb', 'Wo', 'Aq', 'Ak', 'Av', 'Ao', 'cq', 'ck', 'cv',
             'A_log', 'dt_bias', 'o_norm_w')
    return {n: getattr(block, n).detach().float().cpu() for n in names}
