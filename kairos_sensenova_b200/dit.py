"""The Kairos DiT denoise step (``KairosDiT.forward``, ``kairos/modules/dits/kairos_dit.py:1057-1266``)
on this library's kernels, sequence-parallel over P ranks.

Per block (``DiTBlock.forward``, ``kairos_dit.py:823-972``):

    y  = LN(x) * (1 + scale_msa) + shift_msa
    x += gate_msa * mixer(y)                      GatedDeltaNet or FP8 softmax attention (Ulysses)
    y  = LN_affine(x);  x += cross_attn(y, ctx)   q/k RMSNorm, softmax over the text tokens
    y  = LN(x) * (1 + scale_ffn) + shift_ffn
    x += gate_ffn * W2 act(W1 y + b1) + b2

with the six modulation vectors ``modulation + t_mod`` in the reference's order
(scale_msa, shift_msa, gate_msa, scale_ffn, shift_ffn, gate_ffn; ``:874-891,
950-952``).  Every residual add is fused with the LayerNorm and modulation that
follow it (``kb200_residual_ln_mod``): the last one of a block already produces
the next block's (or the head's) modulated input.

Sequence parallelism: rank r owns tokens [r T/P, (r+1) T/P).  Patch embedding,
norms, cross-attention (the 512 text tokens' K/V are computed on every rank),
the FFN and the head are per token; only the mixers exchange data (two
all-to-alls each, :mod:`.mixers`), and the output velocity is all-gathered at
the end of the step.

Model shape: 30 blocks, hidden 3072, 24 heads x 128, FFN
8192 with tanh-GELU, text 512 x 4096, 16-channel latent with 1x2x2 patches.
The mixer pattern is configurable: ``'baseline'`` puts GatedDeltaNet in 3 of
every 4 blocks and softmax attention in every 4th (the benchmark's
description); ``'reference'`` follows ``KairosDiT.__init__`` (``:1125-1134``),
GatedDeltaNet at ``(i + 1) % 4 == 0``.  ``ffn_act='silu'`` gives the
reference's ``ACT2CLS['silu']`` FFN (``:816-819``).  Self-attention is full
(non-causal, no window): the benchmark's attention; the reference's windowed /
dilated variants are not implemented.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .fused_ops import residual_ln_mod, rmsnorm_rope
from .mixers import AttnMixer, GdnMixer


@dataclass
class DiTConfig:
    dim: int = 3072
    heads: int = 24
    ffn_dim: int = 8192
    layers: int = 30
    text_dim: int = 4096
    text_len: int = 512
    freq_dim: int = 256
    in_dim: int = 16
    out_dim: int = 16
    patch: tuple = (1, 2, 2)
    latent: tuple = (21, 60, 104)      # frames, height, width of the latent
    eps: float = 1e-6
    pattern: str = 'baseline'          # 'baseline' | 'reference'
    ffn_act: str = 'gelu_tanh'         # 'gelu_tanh' | 'silu'
    conv_size: int = 4

    @property
    def head_dim(self):
        return self.dim // self.heads

    @property
    def grid(self):
        f, h, w = self.latent
        return f // self.patch[0], h // self.patch[1], w // self.patch[2]

    @property
    def tokens(self):
        f, h, w = self.grid
        return f * h * w

    def is_gdn(self, i):
        if self.pattern == 'reference':
            return (i + 1) % 4 == 0
        return (i + 1) % 4 != 0


def sinusoidal_embedding_1d(dim, position):
    """``kairos/modules/dits/common.py:4-13``: [cos | sin] of position x 10000^(-i/(dim/2)), float64."""
    sinusoid = torch.outer(position.to(torch.float64),
                           torch.pow(10000, -torch.arange(dim // 2, dtype=torch.float64,
                                                          device=position.device).div(dim // 2)))
    return torch.cat([torch.cos(sinusoid), torch.sin(sinusoid)], dim=1)


def make_weights(cfg: DiTConfig, device='cuda', seed=2):
    """Random-init weights of the architecture (bf16 N(0, 0.02) linears and biases,
    ``randn / sqrt(dim)`` modulations as ``DiTBlock.__init__`` :821, GatedDeltaNet's
    A_log / dt_bias init, ``nn.Conv1d``-style uniform short-conv weights, unit
    norm weights), drawn from one seeded device generator so every rank holds
    the same model.  Returns a dict of tensors ([out, in] like ``nn.Linear``)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    bf = torch.bfloat16
    D, H, hd = cfg.dim, cfg.heads, cfg.head_dim
    lin = lambda o, i: (torch.randn(o, i, generator=gen, device=device) * 0.02).to(bf)  # noqa: E731
    bias = lambda o: (torch.randn(o, generator=gen, device=device) * 0.02).to(bf)       # noqa: E731
    ones = lambda n: torch.ones(n, device=device)                                       # noqa: E731
    pin = cfg.in_dim * math.prod(cfg.patch)
    w = {
        'patch_w': lin(D, pin), 'patch_b': bias(D),
        'text_w1': lin(D, cfg.text_dim), 'text_b1': bias(D), 'text_w2': lin(D, D), 'text_b2': bias(D),
        'time_w1': lin(D, cfg.freq_dim), 'time_b1': bias(D), 'time_w2': lin(D, D), 'time_b2': bias(D),
        'tproj_w': lin(6 * D, D), 'tproj_b': bias(6 * D),
        'head_w': lin(cfg.out_dim * math.prod(cfg.patch), D), 'head_b': bias(cfg.out_dim * math.prod(cfg.patch)),
        'head_mod': torch.randn(2, D, generator=gen, device=device) / D ** 0.5,
        'blocks': [],
    }
    bound = 1.0 / math.sqrt(cfg.conv_size)
    for i in range(cfg.layers):
        b = {'mod': torch.randn(6, D, generator=gen, device=device) / D ** 0.5}
        if cfg.is_gdn(i):
            b.update(Wq=lin(D, D), Wk=lin(D, D), Wv=lin(D, D), Wg=lin(D, D), Wa=lin(H, D), Wb=lin(H, D),
                     Wo=lin(D, D), o_norm_w=ones(hd))
            for n in ('cq', 'ck', 'cv'):
                b[n] = (torch.rand(D, cfg.conv_size, generator=gen, device=device) * 2 - 1) * bound
            b['A_log'] = torch.log(torch.rand(H, generator=gen, device=device) * 16).float()
            dt = torch.exp(torch.rand(H, generator=gen, device=device) * (math.log(0.1) - math.log(0.001))
                           + math.log(0.001)).clamp(min=1e-4)
            b['dt_bias'] = (dt + torch.log(-torch.expm1(-dt))).float()
        else:
            b.update(Aq=lin(D, D), Ak=lin(D, D), Av=lin(D, D), Ao=lin(D, D),
                     Abq=bias(D), Abk=bias(D), Abv=bias(D), Abo=bias(D), nq=ones(D), nk=ones(D))
        b.update(Cq=lin(D, D), Ck=lin(D, D), Cv=lin(D, D), Co=lin(D, D), Cbq=bias(D), Cbk=bias(D), Cbv=bias(D),
                 Cbo=bias(D), Cnq=ones(D), Cnk=ones(D), ca_w=ones(D), ca_b=torch.zeros(D, device=device),
                 W1=lin(cfg.ffn_dim, D), b1=bias(cfg.ffn_dim), W2=lin(D, cfg.ffn_dim), b2=bias(D))
        w['blocks'].append(b)
    return w


class _Block:
    def __init__(self, cfg, b, gdn, world, rank, group):
        self.gdn = gdn
        self.mod = b['mod']
        hd = cfg.head_dim
        if gdn:
            self.mixer = GdnMixer(b['Wq'], b['Wk'], b['Wv'], b['Wa'], b['Wb'], b['Wg'], b['Wo'], b['cq'], b['ck'],
                                  b['cv'], b['A_log'], b['dt_bias'], b['o_norm_w'], cfg.heads, hd, world, rank,
                                  group, cfg.eps)
        else:
            self.mixer = AttnMixer(b['Aq'], b['Ak'], b['Av'], b['Ao'], b['nq'], b['nk'], cfg.heads, hd, world,
                                   rank, group, cfg.eps, bq=b['Abq'], bk=b['Abk'], bv=b['Abv'], bo=b['Abo'],
                                   grid=cfg.grid)
        t = lambda W: W.t().contiguous()  # noqa: E731
        self.CqT, self.CkT, self.CvT, self.CoT = t(b['Cq']), t(b['Ck']), t(b['Cv']), t(b['Co'])
        self.Cbq, self.Cbk, self.Cbv, self.Cbo = b['Cbq'], b['Cbk'], b['Cbv'], b['Cbo']
        self.Cnq, self.Cnk = b['Cnq'], b['Cnk']
        self.ca_w, self.ca_b = b['ca_w'], b['ca_b']
        self.W1T, self.b1, self.W2T, self.b2 = t(b['W1']), b['b1'], t(b['W2']), b['b2']


class KairosDiT:
    """B200 denoise step.  ``forward(latent, timestep, context)`` with the full
    latent ``[in_dim, F, H, W]`` and text ``[text_len, text_dim]`` on every rank
    returns the full velocity ``[out_dim, F, H, W]`` (bf16) on every rank."""

    def __init__(self, cfg: DiTConfig, world=1, rank=0, group=None, device='cuda', seed=2, weights=None):
        self.cfg, self.P, self.rank, self.group = cfg, world, rank, group
        if cfg.tokens % world:
            raise ValueError(f'{cfg.tokens} tokens do not split evenly over {world} ranks')
        w = make_weights(cfg, device, seed) if weights is None else weights
        self.w = {k: v for k, v in w.items() if k != 'blocks'}
        self.blocks = [_Block(cfg, b, cfg.is_gdn(i), world, rank, group) for i, b in enumerate(w['blocks'])]
        self.mods = torch.stack([b.mod for b in self.blocks]).float()     # [L, 6, D]
        self._head_wT = self.w['head_w'].t().contiguous()

    # ----------------------------------------------------------------- pieces
    def _patchify(self, latent):
        """[C, F, H, W] -> this rank's patch rows [T/P, C * prod(patch)] (Conv3d
        ``patch_embedding`` as a GEMM: each token's patch flattened as (c, pf, ph, pw))."""
        C, Fr, Hh, Ww = latent.shape
        pf, ph, pw = self.cfg.patch
        x = latent.reshape(C, Fr // pf, pf, Hh // ph, ph, Ww // pw, pw).permute(1, 3, 5, 0, 2, 4, 6)
        Tl = self.cfg.tokens // self.P
        return x.reshape(self.cfg.tokens, -1)[self.rank * Tl:(self.rank + 1) * Tl].to(torch.bfloat16).contiguous()

    def _unpatchify(self, y):
        """[T, (pf ph pw c)] -> [c, F, H, W] (``KairosDiT.unpatchify``, :1176-1181)."""
        f, h, w = self.cfg.grid
        pf, ph, pw = self.cfg.patch
        c = self.cfg.out_dim
        return y.reshape(f, h, w, pf, ph, pw, c).permute(6, 0, 3, 1, 4, 2, 5).reshape(c, f * pf, h * ph, w * pw)

    def _cross(self, blk, y, ctx):
        """``CrossAttention.forward`` (:681-694): q = RMSNorm(W_q y), k = RMSNorm(W_k ctx),
        v = W_v ctx, softmax attention over the text tokens, output projection."""
        cfg = self.cfg
        Tl, H, hd = y.shape[0], cfg.heads, cfg.head_dim
        q = torch.addmm(blk.Cbq, y, blk.CqT)
        rmsnorm_rope(q, blk.Cnq, None, hd, eps=cfg.eps, out=q)
        k = torch.addmm(blk.Cbk, ctx, blk.CkT)
        rmsnorm_rope(k, blk.Cnk, None, hd, eps=cfg.eps, out=k)
        v = torch.addmm(blk.Cbv, ctx, blk.CvT)
        Lc = ctx.shape[0]
        o = F.scaled_dot_product_attention(q.view(1, Tl, H, hd).transpose(1, 2), k.view(1, Lc, H, hd).transpose(1, 2),
                                           v.view(1, Lc, H, hd).transpose(1, 2))
        o = o.transpose(1, 2).reshape(Tl, H * hd)
        return torch.addmm(blk.Cbo, o, blk.CoT)

    def _ffn(self, blk, y):
        if self.cfg.ffn_act == 'gelu_tanh':
            h = torch._addmm_activation(blk.b1, y, blk.W1T, use_gelu=True)
        else:
            h = F.silu(torch.addmm(blk.b1, y, blk.W1T))
        return torch.addmm(blk.b2, h, blk.W2T)

    # ---------------------------------------------------------------- forward
    def forward(self, latent, timestep, context):
        cfg, w = self.cfg, self.w
        eps = cfg.eps
        # time / text embeddings (tiny; torch)
        t_in = sinusoidal_embedding_1d(cfg.freq_dim, timestep.reshape(-1)).to(torch.bfloat16)
        t = torch.addmm(w['time_b2'], F.silu(torch.addmm(w['time_b1'], t_in, w['time_w1'].t())), w['time_w2'].t())
        t_mod = torch.addmm(w['tproj_b'], F.silu(t), w['tproj_w'].t()).float().reshape(6, cfg.dim)
        mods = self.mods + t_mod                                                  # [L, 6, D] fp32
        ctx = context.to(torch.bfloat16)
        ctx = torch.addmm(w['text_b2'], F.silu(torch.addmm(w['text_b1'], ctx, w['text_w1'].t())), w['text_w2'].t())
        # patch embedding of this rank's tokens
        x = torch.addmm(w['patch_b'], self._patchify(latent), w['patch_w'].t())  # residual stream [Tl, D] bf16
        y = torch.empty_like(x)
        m0 = mods[0]
        residual_ln_mod(x, None, None, m0[0], m0[1], True, eps, out=y)
        hm = (w['head_mod'] + t.float()).contiguous()                            # (shift, scale)
        for i, blk in enumerate(self.blocks):
            m = mods[i]
            mix = blk.mixer(y)
            residual_ln_mod(x, mix, m[2], blk.ca_w, blk.ca_b, False, eps, out=y)
            c = self._cross(blk, y, ctx)
            residual_ln_mod(x, c, None, m[3], m[4], True, eps, out=y)
            f = self._ffn(blk, y)
            nscale, nshift = (mods[i + 1][0], mods[i + 1][1]) if i + 1 < len(self.blocks) else (hm[1], hm[0])
            residual_ln_mod(x, f, m[5], nscale, nshift, True, eps, out=y)
        out = torch.addmm(w['head_b'], y, self._head_wT)                          # [Tl, out * prod(patch)]
        if self.P > 1:
            full = torch.empty(self.P * out.shape[0], out.shape[1], device=out.device, dtype=out.dtype)
            dist.all_gather_into_tensor(full, out, group=self.group)
            out = full
        return self._unpatchify(out)

    __call__ = forward

    def launches_per_step(self):
        """Kernel launches of this library per forward() (as of the last call)."""
        n = 1 + 3 * len(self.blocks)                      # residual/LN/modulate sites
        n += 2 * len(self.blocks)                         # cross-attention q and k RMSNorm
        n += sum(b.mixer.launches for b in self.blocks)
        return n
