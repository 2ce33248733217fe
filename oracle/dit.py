"""CPU restatement of the Kairos DiT denoise step (test infrastructure only).

``KairosDiT.forward`` (``kairos/modules/dits/kairos_dit.py:1187-1266``) with
``DiTBlock.forward`` (``:823-972``) in fp32 on the host, for the weights dict of
``kairos_sensenova_b200.dit.make_weights`` and a ``DiTConfig``:

* time / text embeddings (``:1101-1113, 1191-1194``; sinusoid ``common.py:4-13``);
* patch embedding as the Conv3d it is (``:1097, 1167-1174``);
* per block: LayerNorm + modulate (``:306-309, 873-874``), the mixer
  (GatedDeltaNet chain / attention chain, :mod:`oracle.hybrid` and
  ``SelfAttention.forward`` ``:452-479`` with biases), gated residual
  (``:696-701, 929``), cross-attention (``CrossAttention.forward`` ``:681-694``)
  after the affine ``cross_attn_norm``, FFN with its modulation and gate
  (``:950-970``);
* head (``Head.forward`` ``:1047-1052``) and unpatchify (``:1176-1181``).

Only the model pieces are restated here; the GDN and attention arithmetic
comes from :mod:`oracle.gdn` (pinned to the reference's golden vectors) and
torch's SDPA (the reference's own fallback).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .hybrid import freqs_cis_3d, gdn_chain
from .layers import rmsnorm_rope


def _f(t):
    return t.detach().float().cpu()


def _ln(x, eps):
    return F.layer_norm(x, x.shape[-1:], eps=eps)


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _sdpa(q, k, v, H):
    Tq, Tk, D = q.shape[0], k.shape[0], q.shape[1] // H
    o = F.scaled_dot_product_attention(q.reshape(1, Tq, H, D).transpose(1, 2), k.reshape(1, Tk, H, D).transpose(1, 2),
                                       v.reshape(1, Tk, H, D).transpose(1, 2))
    return o.transpose(1, 2).reshape(Tq, H * D)


def self_attention(b, x, H, D, grid, eps):
    """``SelfAttention.forward`` (``kairos_dit.py:452-479``), full attention."""
    T = x.shape[0]
    fr = freqs_cis_3d(D, *grid)
    q = rmsnorm_rope((x @ b['Aq'].t() + b['Abq'])[None], b['nq'], fr, H, eps)[0].float()
    k = rmsnorm_rope((x @ b['Ak'].t() + b['Abk'])[None], b['nk'], fr, H, eps)[0].float()
    v = x @ b['Av'].t() + b['Abv']
    return _sdpa(q, k, v, H) @ b['Ao'].t() + b['Abo']


def cross_attention(b, y, ctx, H, eps):
    q = _rms(y @ b['Cq'].t() + b['Cbq'], b['Cnq'], eps)
    k = _rms(ctx @ b['Ck'].t() + b['Cbk'], b['Cnk'], eps)
    v = ctx @ b['Cv'].t() + b['Cbv']
    return _sdpa(q, k, v, H) @ b['Co'].t() + b['Cbo']


def dit_block(b, x, ctx, t_mod, H, hd, eps, grid, gdn, ffn_act):
    """``DiTBlock.forward`` (``kairos_dit.py:823-972``) for one sequence, fp32:
    x [T, D], ctx [L, D] (already text-embedded), t_mod [6, D]; ``b`` holds the
    block's weights in the layout of ``kairos_sensenova_b200.dit.make_weights``."""
    m = b['mod'] + t_mod                                           # :864-882
    y = _ln(x, eps) * (1 + m[0]) + m[1]                            # scale_msa, shift_msa: :873-874
    if gdn:
        mix = gdn_chain(b, y, H, hd, eps)
    else:
        mix = self_attention(b, y, H, hd, grid, eps)
    x = x + m[2] * mix                                             # gate_msa: :929
    x = x + cross_attention(b, _ln(x, eps) * b['ca_w'] + b['ca_b'], ctx, H, eps)   # :931-933
    y = _ln(x, eps) * (1 + m[3]) + m[4]                            # scale, shift: :950-957
    h = y @ b['W1'].t() + b['b1']
    h = F.gelu(h, approximate='tanh') if ffn_act == 'gelu_tanh' else F.silu(h)
    return x + m[5] * (h @ b['W2'].t() + b['b2'])                 # gate: :958-968


REFERENCE_BLOCK_KEYS = {
    'modulation': 'mod',
    'self_attn.q.weight': 'Aq', 'self_attn.q.bias': 'Abq', 'self_attn.k.weight': 'Ak', 'self_attn.k.bias': 'Abk',
    'self_attn.v.weight': 'Av', 'self_attn.v.bias': 'Abv', 'self_attn.o.weight': 'Ao', 'self_attn.o.bias': 'Abo',
    'self_attn.norm_q.weight': 'nq', 'self_attn.norm_k.weight': 'nk',
    'cross_attn.q.weight': 'Cq', 'cross_attn.q.bias': 'Cbq', 'cross_attn.k.weight': 'Ck', 'cross_attn.k.bias': 'Cbk',
    'cross_attn.v.weight': 'Cv', 'cross_attn.v.bias': 'Cbv', 'cross_attn.o.weight': 'Co', 'cross_attn.o.bias': 'Cbo',
    'cross_attn.norm_q.weight': 'Cnq', 'cross_attn.norm_k.weight': 'Cnk',
    'cross_attn_norm.weight': 'ca_w', 'cross_attn_norm.bias': 'ca_b',
    'ffn.0.weight': 'W1', 'ffn.0.bias': 'b1', 'ffn.2.weight': 'W2', 'ffn.2.bias': 'b2',
}


def block_weights_from_reference(state_dict):
    """A reference ``DiTBlock`` state dict (softmax-attention block) in the
    layout of ``make_weights``'s per-block dicts."""
    b = {REFERENCE_BLOCK_KEYS[k]: v for k, v in state_dict.items() if k in REFERENCE_BLOCK_KEYS}
    b['mod'] = b['mod'].reshape(6, -1)
    return b


def dit_forward(weights, cfg, latent, timestep, context):
    """latent [in_dim, F, H, W], timestep [1], context [text_len, text_dim] -> [out_dim, F, H, W] fp32."""
    w = {k: _f(v) for k, v in weights.items() if k != 'blocks'}
    D, H, hd, eps = cfg.dim, cfg.heads, cfg.head_dim, cfg.eps
    half = cfg.freq_dim // 2
    pos = timestep.double().cpu().reshape(-1)
    s = torch.outer(pos, torch.pow(10000, -torch.arange(half, dtype=torch.float64).div(half)))
    t_in = torch.cat([torch.cos(s), torch.sin(s)], 1).float()
    t = F.silu(t_in @ w['time_w1'].t() + w['time_b1']) @ w['time_w2'].t() + w['time_b2']
    t_mod = (F.silu(t) @ w['tproj_w'].t() + w['tproj_b']).reshape(6, D)
    ctx = _f(context)
    ctx = F.silu(ctx @ w['text_w1'].t() + w['text_b1']) @ w['text_w2'].t() + w['text_b2']
    pf, ph, pw = cfg.patch
    conv_w = w['patch_w'].reshape(D, cfg.in_dim, pf, ph, pw)
    x = F.conv3d(_f(latent)[None], conv_w, w['patch_b'], stride=cfg.patch)[0]      # [D, f, h, w]
    grid = x.shape[1:]
    x = x.flatten(1).t()                                                             # [T, D]
    for i, braw in enumerate(weights['blocks']):
        b = {k: _f(v) for k, v in braw.items()}
        x = dit_block(b, x, ctx, t_mod, H, hd, eps, tuple(grid), cfg.is_gdn(i), cfg.ffn_act)
    shift, scale = w['head_mod'] + t
    out = (_ln(x, eps) * (1 + scale) + shift) @ w['head_w'].t() + w['head_b']        # [T, pf ph pw c]
    f_, h_, w_ = grid
    c = cfg.out_dim
    return out.reshape(f_, h_, w_, pf, ph, pw, c).permute(6, 0, 3, 1, 4, 2, 5).reshape(c, f_ * pf, h_ * ph, w_ * pw)


def tokens_of(cfg):
    return math.prod(cfg.grid)


def self_attention_rows(b, x, H, D, grid, eps, rows):
    """``self_attention`` for the query rows ``[0, rows)`` only (keys and values
    from every token): the exact values of those rows at a fraction of the cost."""
    fr = freqs_cis_3d(D, *grid)
    q = rmsnorm_rope((x[:rows] @ b['Aq'].t() + b['Abq'])[None], b['nq'], fr[:rows], H, eps)[0].float()
    k = rmsnorm_rope((x @ b['Ak'].t() + b['Abk'])[None], b['nk'], fr, H, eps)[0].float()
    v = x @ b['Av'].t() + b['Abv']
    return _sdpa(q, k, v, H) @ b['Ao'].t() + b['Abo']


def dit_forward_rows(weights, cfg, latent, timestep, context, rows):
    """A ONE-block model (``cfg.layers == 1``) for the first ``rows`` tokens only:
    returns the head output ``[rows, pf*ph*pw*out_dim]`` before unpatchify.
    Exact for those rows -- everything but the mixer is per token, the
    GatedDeltaNet mixer is causal (a prefix needs only the prefix) and the
    attention mixer takes its keys and values from every token -- so a
    full-size block can be checked without the full-sequence CPU cost."""
    assert cfg.layers == 1
    w = {k: _f(v) for k, v in weights.items() if k != 'blocks'}
    D, H, hd, eps = cfg.dim, cfg.heads, cfg.head_dim, cfg.eps
    half = cfg.freq_dim // 2
    pos = timestep.double().cpu().reshape(-1)
    s = torch.outer(pos, torch.pow(10000, -torch.arange(half, dtype=torch.float64).div(half)))
    t_in = torch.cat([torch.cos(s), torch.sin(s)], 1).float()
    t = F.silu(t_in @ w['time_w1'].t() + w['time_b1']) @ w['time_w2'].t() + w['time_b2']
    t_mod = (F.silu(t) @ w['tproj_w'].t() + w['tproj_b']).reshape(6, D)
    ctx = _f(context)
    ctx = F.silu(ctx @ w['text_w1'].t() + w['text_b1']) @ w['text_w2'].t() + w['text_b2']
    pf, ph, pw = cfg.patch
    conv_w = w['patch_w'].reshape(D, cfg.in_dim, pf, ph, pw)
    x = F.conv3d(_f(latent)[None], conv_w, w['patch_b'], stride=cfg.patch)[0]
    grid = tuple(x.shape[1:])
    x = x.flatten(1).t()                                                             # [T, D]
    b = {k: _f(v) for k, v in weights['blocks'][0].items()}
    m = b['mod'] + t_mod
    gdn = cfg.is_gdn(0)
    y = _ln(x if not gdn else x[:rows], eps) * (1 + m[0]) + m[1]
    mix = gdn_chain(b, y, H, hd, eps) if gdn else self_attention_rows(b, y, H, hd, grid, eps, rows)
    x = x[:rows] + m[2] * mix
    x = x + cross_attention(b, _ln(x, eps) * b['ca_w'] + b['ca_b'], ctx, H, eps)
    y = _ln(x, eps) * (1 + m[3]) + m[4]
    h = y @ b['W1'].t() + b['b1']
    h = F.gelu(h, approximate='tanh') if cfg.ffn_act == 'gelu_tanh' else F.silu(h)
    x = x + m[5] * (h @ b['W2'].t() + b['b2'])
    shift, scale = w['head_mod'] + t
    return (_ln(x, eps) * (1 + scale) + shift) @ w['head_w'].t() + w['head_b']


def patch_rows(velocity, cfg):
    """Inverse of unpatchify: ``[c, F, H, W]`` -> ``[T, pf*ph*pw*c]`` token rows."""
    f, h, w = cfg.grid
    pf, ph, pw = cfg.patch
    c = velocity.shape[0]
    return velocity.reshape(c, f, pf, h, ph, w, pw).permute(1, 3, 5, 2, 4, 6, 0).reshape(f * h * w, -1)
