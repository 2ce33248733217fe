"""Token mixers of the Kairos DiT, Ulysses-sharded over P ranks.

Per rank the input is a sequence shard ``x_local [T/P, hidden]`` (bf16).

:class:`GdnMixer` -- the GatedDeltaNet half of ``DiTBlock.forward``
(``kairos_dit.py:858-928``; layer ``fla/layers/gated_deltanet.py:234-315``),
re-partitioned Ulysses-style instead of the reference's per-owner broadcast:
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

:class:`AttnMixer` -- ``SelfAttention`` / ``SelfAttentionTP.forward``
(``kairos_dit.py:452-479, 603-650``): q|k|v projection grouped by destination,
q and k full-dimension RMSNorm + 3-D RoPE in place in the projection buffer
before the exchange (one fused kernel, ``kairos_dit.py:452-456``), seq->head
all-to-all, FP8 attention on the rank's heads, head->seq all-to-all, ``o``
projection.  Biases (``nn.Linear`` in the DiT) are optional.

Each mixer keeps only its destination-packed weights; the caller may drop the
full-size ones after construction.
"""
from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist

from .attention import attention_fp8
from .fused_ops import freqs_cis_3d, gdn_prologue, rms_norm_gated, rmsnorm_rope, rope_table
from .gated_delta_rule import chunk_gated_delta_rule


def _round8(n):
    return (n + 7) // 8 * 8


def _marker(phases, prefix):
    """A function recording a CUDA event named ``prefix.name`` on the current stream
    into ``phases`` (a no-op when ``phases`` is None)."""
    if phases is None:
        return lambda name: None

    def mark(name):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        phases.append((f'{prefix}.{name}', e))
    return mark


_COMM_STREAMS = {}


def _comm_stream(dev):
    s = _COMM_STREAMS.get(dev)
    if s is None:
        s = _COMM_STREAMS[dev] = torch.cuda.Stream(dev)
    return s


class _Ulysses:
    # token slabs of the seq->head exchange: the projection GEMM of slab i+1 runs
    # while slab i crosses NVLink (0 = choose from the shard size)
    slabs = 0

    def __init__(self, heads, head_dim, world, rank, group):
        if heads % world:
            raise ValueError('heads must divide evenly over ranks')
        self.H, self.D, self.P, self.rank, self.group = heads, head_dim, world, rank, group
        self.Hl = heads // world

    def _project_exchange(self, x_local, W, b, post=None):
        """Projection grouped by destination + seq->head exchange: returns
        ``[T, C]`` (all tokens of this rank's heads, in token order).

        With P > 1 the rows of the shard are processed in slabs: the GEMM of
        a slab writes ``[P, n, C]`` (destination-major, so each destination's
        part is contiguous), ``post`` (if given) transforms it in place, and
        grouped NCCL sends/receives on a side stream move it while the next
        slab is projected.  Rank ``src``'s rows ``[r0, r0+n)`` land in rows
        ``src * T/P + r0 ..`` of the result, which is therefore already in
        global token order."""
        Tl = x_local.shape[0]
        C = W.shape[-1]
        if self.P == 1:
            send = self._project(x_local, W, b)
            if post is not None:
                post(send, 0)
            return send.reshape(Tl, C)
        P, rank = self.P, self.rank
        # auto: one slab for short shards (at 8 GPUs, 4095 rows: one slab 2.53 ms per
        # graph-replayed hybrid step against 2.58 with three and 2.60 with two), else up to 4
        ns = self.slabs or (1 if Tl <= 4096 else min(4, Tl // 1024))
        step = -(-Tl // ns)
        recv = torch.empty(P, Tl, C, device=x_local.device, dtype=x_local.dtype)
        cuda = x_local.is_cuda          # (CPU tensors: the gloo tests of the data layout)
        comp = torch.cuda.current_stream(x_local.device) if cuda else None
        comm = _comm_stream(x_local.device) if cuda else None
        for r0 in range(0, Tl, step):
            r1 = min(Tl, r0 + step)
            send = self._project(x_local[r0:r1], W, b)                 # [P, n, C]
            if post is not None:
                post(send, r0)
            if cuda:
                comm.wait_stream(comp)
            with torch.cuda.stream(comm) if cuda else contextlib.nullcontext():
                ops = []
                for peer in range(P):
                    if peer != rank:
                        ops.append(dist.P2POp(dist.isend, send[peer], self._global(peer), self.group))
                        ops.append(dist.P2POp(dist.irecv, recv[peer, r0:r1], self._global(peer), self.group))
                for req in dist.batch_isend_irecv(ops):
                    req.wait()
                recv[rank, r0:r1].copy_(send[rank])
            if cuda:
                send.record_stream(comm)
        if cuda:
            comp.wait_stream(comm)
        return recv.reshape(P * Tl, C)

    def _global(self, peer):
        return peer if self.group is None else dist.get_global_rank(self.group, peer)

    def _rows(self, W, r, d):
        return W[r * self.Hl * d:(r + 1) * self.Hl * d]

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

    def _project(self, x_local, W, b):
        """[Tl, hidden] -> [P, Tl, C] grouped by destination rank (+ bias)."""
        if b is None:
            return torch.matmul(x_local.unsqueeze(0), W)
        if self.P == 1:   # the bias in cuBLASLt's epilogue
            return torch.addmm(b[0], x_local, W[0]).unsqueeze(0)
        out = torch.matmul(x_local.unsqueeze(0), W)
        out += b.unsqueeze(1)
        return out


class GdnMixer(_Ulysses):
    """Weights as ``nn.Linear`` ([out, in]); ``A_log``/``dt_bias`` [H]; conv [H*D, W]."""

    # kernel launches of this library per call: prologue, GDN (3, or 5 when the
    # state pass is segmented; updated by each call), gated RMSNorm
    launches = 5

    def __init__(self, Wq, Wk, Wv, Wa, Wb, Wg, Wo, cq, ck, cv, A_log, dt_bias, o_norm_w, heads, head_dim,
                 world=1, rank=0, group=None, eps=1e-5):
        super().__init__(heads, head_dim, world, rank, group)
        P, Hl, D = self.P, self.Hl, self.D
        self.eps = eps
        self.C = _round8(3 * Hl * D + 2 * Hl)
        blocks = []
        for r in range(P):
            blk = torch.cat([self._rows(Wq, r, D), self._rows(Wk, r, D), self._rows(Wv, r, D),
                             self._rows(Wa, r, 1), self._rows(Wb, r, 1)])
            pad = self.C - blk.shape[0]
            if pad:
                blk = torch.cat([blk, blk.new_zeros(pad, blk.shape[1])])
            blocks.append(blk.t())
        self.W = torch.stack(blocks).contiguous()      # [P, hidden, C]
        sl = slice(rank * Hl * D, (rank + 1) * Hl * D)
        self.cq, self.ck, self.cv = cq[sl].contiguous(), ck[sl].contiguous(), cv[sl].contiguous()
        hs = slice(rank * Hl, (rank + 1) * Hl)
        self.A_log, self.dt_bias = A_log[hs].contiguous(), dt_bias[hs].contiguous()
        self.WgT = Wg.t().contiguous()
        self.WoT = Wo.t().contiguous()
        self.o_norm_w = o_norm_w

    def __call__(self, x_local, phases=None):
        """``phases`` (optional list) receives (name, CUDA event) marks at the phase
        boundaries on the compute stream: projection + seq->head exchange, prologue,
        GDN, head->seq exchange, epilogue (gate, norm, o_proj)."""
        mark = _marker(phases, 'gdn')
        Tl = x_local.shape[0]
        T = Tl * self.P
        Hl, D = self.Hl, self.D
        mark('start')
        recv = self._project_exchange(x_local, self.W, None)            # [T, C]
        mark('proj_exchange')
        c = lambda i: recv[:, i * Hl * D:(i + 1) * Hl * D]  # noqa: E731
        ab = 3 * Hl * D
        q, k, v, g, beta = gdn_prologue(c(0), c(1), c(2), recv[:, ab:ab + Hl], recv[:, ab + Hl:ab + 2 * Hl],
                                        self.cq, self.ck, self.cv, self.A_log, self.dt_bias, Hl, 1, T)
        mark('prologue')
        o, _ = chunk_gated_delta_rule(q, k, v, g, beta, use_qk_l2norm_in_kernel=True)
        mark('gdn')
        self.launches = 2 + chunk_gated_delta_rule.launches
        o_seq = self._head_to_seq(o.reshape(T, Hl * D), Tl)
        mark('head_to_seq')
        gate = x_local @ self.WgT
        y = rms_norm_gated(o_seq.reshape(Tl, self.H, D), gate.reshape(Tl, self.H, D), self.o_norm_w, self.eps)
        out = y.reshape(Tl, -1) @ self.WoT
        mark('epilogue')
        return out


class AttnMixer(_Ulysses):
    """Weights as ``nn.Linear`` ([out, in]), optional biases; ``nq``/``nk``: the
    full-dimension RMSNorm weights; ``grid``: the (frames, height, width) latent
    grid of the 3-D RoPE (a 1-D axis when it does not hold T tokens)."""

    # q and k RMSNorm+RoPE per exchange slab, amax, quantise, attention (updated by each call)
    launches = 5

    def __init__(self, Wq, Wk, Wv, Wo, nq, nk, heads, head_dim, world=1, rank=0, group=None, eps=1e-6,
                 bq=None, bk=None, bv=None, bo=None, grid=None):
        super().__init__(heads, head_dim, world, rank, group)
        P, Hl, D = self.P, self.Hl, self.D
        self.eps, self.grid, self._rope = eps, grid, None
        self.C = 3 * Hl * D
        self.W = torch.stack([torch.cat([self._rows(Wq, r, D), self._rows(Wk, r, D), self._rows(Wv, r, D)]).t()
                              for r in range(P)]).contiguous()          # [P, hidden, C]
        self.b = None
        if bq is not None:
            self.b = torch.stack([torch.cat([self._rows(bq, r, D), self._rows(bk, r, D), self._rows(bv, r, D)])
                                  for r in range(P)]).contiguous()      # [P, C]
        self.WoT = Wo.t().contiguous()
        self.bo = bo
        self.nq, self.nk = nq, nk

    def rope(self, T):
        """(cos, sin) table [T, D/2, 2] of the 3-D RoPE grid."""
        if self._rope is None or self._rope.shape[0] != T:
            g = self.grid
            f, h, w = g if g is not None and g[0] * g[1] * g[2] == T else (T, 1, 1)
            self._rope = rope_table(freqs_cis_3d(self.D, f, h, w), self.W.device)
        return self._rope

    def __call__(self, x_local, events=None, phases=None):
        """``events`` (optional start/end pair) brackets the attention kernel;
        ``phases`` (optional list) receives (name, CUDA event) phase marks:
        projection + norm/RoPE + seq->head exchange, attention, head->seq
        exchange, o_proj."""
        mark = _marker(phases, 'attn')
        mark('start')
        Tl = x_local.shape[0]
        T = Tl * self.P
        Hl, D = self.Hl, self.D
        cs = self.rope(T)[self.rank * Tl:(self.rank + 1) * Tl]

        self.launches = 3

        def norm_rope(send, r0):
            # q/k RMSNorm over all heads + RoPE, in place, sequence-sharded (before the exchange)
            self.launches += 2
            n = send.shape[1]
            for col, wgt in ((0, self.nq), (Hl * D, self.nk)):
                view = send[..., col:]
                rmsnorm_rope(view, wgt, cs[r0:r0 + n], D, eps=self.eps, out=view, rows=n, dim=self.H * D,
                             ld=self.C, heads_per_block=Hl, block_stride=n * self.C)

        recv = self._project_exchange(x_local, self.W, self.b, norm_rope)  # [T, 3*Hl*D]
        mark('proj_exchange')
        q, k, v = (recv[:, i * Hl * D:(i + 1) * Hl * D].reshape(1, T, Hl * D) for i in range(3))
        o = attention_fp8(q, k, v, Hl, events=events)
        mark('attention')
        o_seq = self._head_to_seq(o.reshape(T, Hl * D), Tl)
        mark('head_to_seq')
        out = o_seq @ self.WoT if self.bo is None else torch.addmm(self.bo, o_seq, self.WoT)
        mark('o_proj')
        return out
