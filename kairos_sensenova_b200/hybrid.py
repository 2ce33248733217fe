"""The sequence-parallel hybrid block of the benchmark: one
GDN mixer chain and one FP8-attention mixer chain, Ulysses-sharded over P
ranks (the chains themselves are :mod:`.mixers`).

Per rank the input is a sequence shard ``x_local [T/P, hidden]`` (bf16).
Weights are drawn on the device from a seeded generator, identically on every
rank; the full-size copies stay on the block so that tests can hand them to
the CPU oracle.
"""
from __future__ import annotations

import math

import torch

from .mixers import AttnMixer, GdnMixer


class HybridBlock:
    def __init__(self, hidden=3072, heads=24, head_dim=128, world=1, rank=0, group=None,
                 device='cuda', seed=3, conv_size=4, norm_eps=1e-5, grid=(21, 30, 52),
                 attn_eps=1e-6):
        assert heads % world == 0, 'heads must divide evenly over ranks'
        self.hidden, self.H, self.D = hidden, heads, head_dim
        self.P, self.rank, self.group = world, rank, group
        self.Hl = heads // world
        self.eps = norm_eps
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)          # identical weights on every rank
        bf = torch.bfloat16
        w = lambda *s: (torch.randn(*s, generator=gen, device=device) * 0.02).to(bf)  # noqa: E731
        HD = heads * head_dim
        # full-size weights (as the reference's nn.Linear weights, [out, in])
        self.Wq, self.Wk, self.Wv, self.Wg = w(HD, hidden), w(HD, hidden), w(HD, hidden), w(HD, hidden)
        self.Wa, self.Wb = w(heads, hidden), w(heads, hidden)
        self.Wo = w(hidden, HD)
        self.Aq, self.Ak, self.Av, self.Ao = w(HD, hidden), w(HD, hidden), w(HD, hidden), w(hidden, HD)
        # ShortConvolution weights: nn.Conv1d default init U(-1/sqrt(W), 1/sqrt(W)) under the seed
        bound = 1.0 / math.sqrt(conv_size)
        cw = lambda c: ((torch.rand(c, conv_size, generator=gen, device=device) * 2 - 1) * bound)  # noqa: E731
        self.cq, self.ck, self.cv = cw(HD), cw(HD), cw(HD)
        # A_log, dt_bias as GatedDeltaNet.__init__ (gated_deltanet.py:151-165)
        self.A_log = torch.log(torch.rand(heads, generator=gen, device=device) * 16).float()
        dt = torch.exp(torch.rand(heads, generator=gen, device=device) * (math.log(0.1) - math.log(0.001))
                       + math.log(0.001)).clamp(min=1e-4)
        self.dt_bias = (dt + torch.log(-torch.expm1(-dt))).float()
        self.o_norm_w = torch.ones(head_dim, device=device)
        # attention q/k RMSNorm weights (FusedRMSNorm init: ones) and the 3-D RoPE grid
        self.nq = torch.ones(HD, device=device)
        self.nk = torch.ones(HD, device=device)
        self.grid, self.attn_eps = grid, attn_eps
        self.gdn = GdnMixer(self.Wq, self.Wk, self.Wv, self.Wa, self.Wb, self.Wg, self.Wo, self.cq, self.ck,
                            self.cv, self.A_log, self.dt_bias, self.o_norm_w, heads, head_dim, world, rank,
                            group, norm_eps)
        self.attn = AttnMixer(self.Aq, self.Ak, self.Av, self.Ao, self.nq, self.nk, heads, head_dim, world,
                              rank, group, attn_eps, grid=grid)

    def gdn_chain(self, x_local, phases=None):
        return self.gdn(x_local, phases=phases)

    def attn_chain(self, x_local, events=None, phases=None):
        return self.attn(x_local, events, phases=phases)

    def forward(self, x_local, events=None, phases=None):
        """One hybrid step: the GDN chain, then the attention chain on its output.
        ``events`` (optional start/end pair) brackets the attention kernel;
        ``phases`` (optional list) collects per-phase CUDA event marks."""
        y = self.gdn_chain(x_local, phases)
        return self.attn_chain(y, events, phases)

    def launches_per_step(self):
        """Kernel launches of this library per forward() (as of the last call)."""
        return self.gdn.launches + self.attn.launches
