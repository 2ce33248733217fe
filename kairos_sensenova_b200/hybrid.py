"""The sequence-parallel hybrid block of the benchmark (one GDN mixer chain
and one FP8-attention mixer chain), Ulysses-sharded over P ranks.

Per rank the input is a sequence shard ``x_local [T/P, hidden]`` (bf16).

GDN chain (the GDN half of ``DiTBlock.forward``, ``kairos_dit.py:858-928``,
re-partitioned Ulysses-style instead of the reference's per-owner broadcast):
  1. one batched projection GEMM writes q|k|v|a|b already grouped by
     destination rank: ``[P, T/P, C_loc]`` (cuBLAS);
  2. ``all_to_all_single`` seq->head: every rank gets all T tokens of its
     ``H/P`` heads (NCCL over NVLink);
  3. prologue kernel: short convs + SiLU, beta, g (the causal conv needs the
     full sequence of a head, which the rank now holds -- no halo exchange);
  4. chunked GDN kernels;
  5. ``all_to_all_single`` head->seq;
  6. epilogue kernel: gated RMSNorm with ``g_proj(x_local)`` (seq-sharded, so
     the gate never crosses the wire), then ``o_proj``.

Attention chain (``SelfAttentionTP.forward``, ``kairos_dit.py:603-650``):
  q|k|v projection grouped by destination, seq->head all-to-all, FP8
  attention on the rank's heads, head->seq all-to-all, ``o`` projection.
  q and k get the layer's full-dimension RMSNorm and 3-D RoPE in place in the
  projection buffer before the exchange (one fused kernel, ``kairos_dit.py:452-456``).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .attention import attention_fp8
from .fused_ops import freqs_cis_3d, gdn_prologue, rms_norm_gated, rmsnorm_rope, rope_table
from .gated_delta_rule import chunk_gated_delta_rule


def _round8(n):
    return (n + 7) // 8 * 8


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
        self.grid, self.attn_eps, self._rope = grid, attn_eps, None
        self._pack()

    # ------------------------------------------------------------------ layout
    def _pack(self):
        """Group projection columns by destination rank (the all-to-all send order)."""
        P, Hl, D = self.P, self.Hl, self.D
        rows = lambda W, r, d: W[r * Hl * d:(r + 1) * Hl * d]  # noqa: E731
        self.C_gdn = _round8(3 * Hl * D + 2 * Hl)
        self.C_attn = 3 * Hl * D
        Wg, Wa = [], []
        for r in range(P):
            blk = torch.cat([rows(self.Wq, r, D), rows(self.Wk, r, D), rows(self.Wv, r, D),
                             rows(self.Wa, r, 1), rows(self.Wb, r, 1)])
            pad = self.C_gdn - blk.shape[0]
            if pad:
                blk = torch.cat([blk, blk.new_zeros(pad, blk.shape[1])])
            Wg.append(blk.t())
            Wa.append(torch.cat([rows(self.Aq, r, D), rows(self.Ak, r, D), rows(self.Av, r, D)]).t())
        self.W_gdn = torch.stack(Wg).contiguous()      # [P, hidden, C_gdn]
        self.W_attn = torch.stack(Wa).contiguous()     # [P, hidden, C_attn]
        sl = slice(self.rank * Hl * D, (self.rank + 1) * Hl * D)
        self.cq_l, self.ck_l, self.cv_l = self.cq[sl], self.ck[sl], self.cv[sl]
        hs = slice(self.rank * Hl, (self.rank + 1) * Hl)
        self.A_log_l, self.dt_bias_l = self.A_log[hs], self.dt_bias[hs]
        self.WgT = self.Wg.t().contiguous()
        self.WoT = self.Wo.t().contiguous()
        self.AoT = self.Ao.t().contiguous()

    def _a2a(self, send):
        if self.P == 1:
            return send
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv

    def _head_to_seq(self, o_heads, Tl):
        """[T, Hl*D] head-sharded -> [Tl, H*D] sequence-sharded."""
        send = o_heads.reshape(self.P, Tl, self.Hl * self.D)
        recv = self._a2a(send)
        return recv.permute(1, 0, 2).reshape(Tl, self.H * self.D) if self.P > 1 else recv.reshape(Tl, -1)

    # ------------------------------------------------------------------ chains
    def gdn_chain(self, x_local):
        Tl = x_local.shape[0]
        T = Tl * self.P
        Hl, D = self.Hl, self.D
        send = torch.matmul(x_local.unsqueeze(0), self.W_gdn)          # [P, Tl, C_gdn]
        recv = self._a2a(send).reshape(T, self.C_gdn)
        c = lambda i: recv[:, i * Hl * D:(i + 1) * Hl * D]  # noqa: E731
        ab = 3 * Hl * D
        q, k, v, g, beta = gdn_prologue(c(0), c(1), c(2), recv[:, ab:ab + Hl], recv[:, ab + Hl:ab + 2 * Hl],
                                        self.cq_l, self.ck_l, self.cv_l, self.A_log_l, self.dt_bias_l,
                                        Hl, 1, T)
        o, _ = chunk_gated_delta_rule(q, k, v, g, beta, use_qk_l2norm_in_kernel=True)
        o_seq = self._head_to_seq(o.reshape(T, Hl * D), Tl)
        gate = x_local @ self.WgT
        y = rms_norm_gated(o_seq.reshape(Tl, self.H, D), gate.reshape(Tl, self.H, D), self.o_norm_w, self.eps)
        return y.reshape(Tl, -1) @ self.WoT

    def rope(self, T):
        """(cos, sin) table [T, D/2, 2] of the 3-D RoPE grid (a 1-D frame axis when
        the grid does not hold T tokens)."""
        if self._rope is None or self._rope.shape[0] != T:
            f, h, w = self.grid if self.grid[0] * self.grid[1] * self.grid[2] == T else (T, 1, 1)
            self._rope = rope_table(freqs_cis_3d(self.D, f, h, w), self.W_attn.device)
        return self._rope

    def attn_chain(self, x_local, events=None):
        Tl = x_local.shape[0]
        T = Tl * self.P
        Hl, D = self.Hl, self.D
        send = torch.matmul(x_local.unsqueeze(0), self.W_attn)          # [P, Tl, 3*Hl*D]
        # q/k RMSNorm over all heads + RoPE, in place, sequence-sharded (before the exchange)
        cs = self.rope(T)[self.rank * Tl:(self.rank + 1) * Tl]
        for col, wgt in ((0, self.nq), (Hl * D, self.nk)):
            view = send[..., col:]
            rmsnorm_rope(view, wgt, cs, D, eps=self.attn_eps, out=view, rows=Tl, dim=self.H * D,
                         ld=self.C_attn, heads_per_block=Hl, block_stride=Tl * self.C_attn)
        recv = self._a2a(send).reshape(T, self.C_attn)
        q, k, v = (recv[:, i * Hl * D:(i + 1) * Hl * D].reshape(1, T, Hl * D) for i in range(3))
        o = attention_fp8(q, k, v, Hl, events=events)
        o_seq = self._head_to_seq(o.reshape(T, Hl * D), Tl)
        return o_seq @ self.AoT

    def forward(self, x_local, events=None):
        """One hybrid step: the GDN chain, then the attention chain on its output.
        ``events`` (optional start/end pair) brackets the attention kernel."""
        y = self.gdn_chain(x_local)
        return self.attn_chain(y, events)

    # kernel launches of this library per forward(): prologue, 3 GDN kernels,
    # gated RMSNorm; q and k RMSNorm+RoPE, amax, quantise, attention
    LAUNCHES_PER_STEP = 10
