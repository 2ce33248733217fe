"""CPU restatement of the gated delta rule forward (test infrastructure only).

Two independent formulations of the same operator:

* :func:`gdn_recurrent` -- the token-by-token recurrence of the reference's
  ``naive_recurrent_gated_delta_product`` with ``num_householder=1``
  (``kairos/third_party/fla/ops/gated_delta_product/naive.py:4-36``).
  Unlike that function it honours ``scale`` and can L2-normalise q/k itself
  (the reference function ignores ``scale``, ``naive.py:4`` vs ``:23-35``).

* :func:`gdn_chunk` -- the chunked algorithm of
  ``chunk_gated_delta_rule_fwd`` (``fla/ops/gated_delta_rule/chunk.py:16-67``)
  phase by phase: local gate cumsum, beta-scaled K K^T, (I+A)^-1, the WY
  vectors w/u, the sequential inter-chunk state pass, and the output combine.
  With ``emulate_bf16=True`` it rounds to bf16 at exactly the points where the
  reference's Triton kernels store or feed a bf16 operand, so that it models
  what a bf16 implementation of the same pipeline should produce.

All arithmetic is torch on CPU in float32 (or float64 if the inputs are).
Layouts follow the reference: q,k ``[B,T,H,K]``, v ``[B,T,H,V]``, g and beta
``[B,T,H]``, states ``[N,H,K,V]``.
"""
from __future__ import annotations

import torch

BT = 64  # chunk size hard-wired by chunk.py:27 (chunk_local_cumsum(..., chunk_size=64))


def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(x.dtype)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """y = x / sqrt(sum(x^2) + eps) over the last dim.

    ``fla/modules/l2norm.py:118-121`` (kernel) and ``:157-160`` (eps default).
    """
    xf = x.float() if x.dtype != torch.float64 else x
    return xf / torch.sqrt((xf * xf).sum(-1, keepdim=True) + eps)


def gdn_recurrent(q, k, v, g, beta, scale=None, initial_state=None,
                  output_final_state=True, use_qk_l2norm=False):
    """Token recurrence; ``naive.py:17-35``.

    For every token t and head:  h <- e^{g_t} h;
    h <- h + beta_t k_t (v_t - h^T k_t)^T;  o_t = scale * h^T q_t.
    Returns (o [B,T,H,V] float, h [B,H,K,V] float or None).
    """
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    q, k, v, g, beta = (x.to(dt) for x in (q, k, v, g, beta))
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    h = torch.zeros(B, H, K, V, dtype=dt)
    if initial_state is not None:
        h = initial_state.to(dt).clone()
    o = torch.zeros(B, T, H, V, dtype=dt)
    for t in range(T):
        h = h * g[:, t].exp()[..., None, None]
        kt, vt, bt = k[:, t], v[:, t], beta[:, t]
        pred = torch.einsum('bhkv,bhk->bhv', h, kt)
        h = h + torch.einsum('bhk,bhv->bhkv', kt, (vt - pred) * bt[..., None])
        o[:, t] = torch.einsum('bhkv,bhk->bhv', h, q[:, t]) * scale
    return o, (h if output_final_state else None)


def chunk_local_cumsum(g: torch.Tensor, T: int) -> torch.Tensor:
    """Inclusive prefix sum of g inside each 64-token chunk, fp32.

    ``fla/ops/utils/cumsum.py:27-65`` (scalar kernel, forward direction).
    g: [B,T,H] -> [B,T,H].
    """
    out = torch.empty_like(g, dtype=torch.float32 if g.dtype != torch.float64 else g.dtype)
    for s in range(0, T, BT):
        e = min(s + BT, T)
        out[:, s:e] = g[:, s:e].to(out.dtype).cumsum(1)
    return out


def _chunks(T):
    return [(s, min(s + BT, T)) for s in range(0, T, BT)]


def scaled_dot_kkt(k, gc, beta, s, e):
    """A[i,j] = beta_i e^{g_i-g_j} <k_i,k_j> for i>j else 0, one chunk.

    ``fla/ops/common/chunk_scaled_dot_kkt.py:51-70``.  The exponent is only
    evaluated where the mask keeps the entry (i>j gives g_i-g_j <= 0), which
    is the same value the reference keeps after its ``tl.where``.
    k: [B,T,H,K] -> A: [B,H,L,L] with L = e-s.
    """
    kc = k[:, s:e].permute(0, 2, 1, 3)                     # B,H,L,K
    A = kc @ kc.transpose(-1, -2)
    gcc = gc[:, s:e].permute(0, 2, 1)                      # B,H,L
    L = e - s
    mask = torch.tril(torch.ones(L, L, dtype=torch.bool), -1)
    diff = (gcc[..., :, None] - gcc[..., None, :]).masked_fill(~mask, 0.0)
    A = A * diff.exp() * beta[:, s:e].permute(0, 2, 1)[..., :, None].to(A.dtype)
    return A.masked_fill(~mask, 0.0)


def solve_tril(A):
    """(I + A)^-1 for strictly lower-triangular A, per chunk.

    ``fla/ops/utils/solve_tril.py:335-382`` (merge_16x16_to_64x64_inverse
    kernel ``:184-331``).  Restated as a plain forward substitution, which is
    exact in the same arithmetic; the reference's 16x16 block merge is an
    evaluation order of the same triangular inverse.
    """
    L = A.shape[-1]
    eye = torch.eye(L, dtype=A.dtype).expand_as(A)
    return torch.linalg.solve_triangular(eye + A, eye.clone(), upper=False, unitriangular=True)


def gdn_chunk(q, k, v, g, beta, scale=None, initial_state=None,
              output_final_state=True, use_qk_l2norm=False, emulate_bf16=False,
              return_intermediates=False):
    """Chunked forward, ``chunk.py:16-67`` plus the l2norm step at ``:166-168``.

    Returns (o [B,T,H,V] float, final_state [B,H,K,V] float or None)
    and, if ``return_intermediates``, a dict with gc, Ai, w, u, v_new, h.
    """
    dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    rnd = _bf16 if emulate_bf16 else (lambda x: x)
    q, k, v, g, beta = (x.to(dt) for x in (q, k, v, g, beta))
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    if use_qk_l2norm:                     # chunk.py:166-168; y stored in input dtype
        q, k = rnd(l2norm(q)), rnd(l2norm(k))
    gc = chunk_local_cumsum(g, T)         # chunk.py:27
    chunks = _chunks(T)
    w = torch.zeros(B, T, H, K, dtype=dt)
    u = torch.zeros(B, T, H, V, dtype=dt)
    Ais = []
    for s, e in chunks:
        A = scaled_dot_kkt(k, gc, beta, s, e)                        # chunk.py:29-35
        Ai = rnd(solve_tril(A))                                      # chunk.py:36-40 (output_dtype=k.dtype)
        Ais.append(Ai)
        bc = beta[:, s:e].permute(0, 2, 1)[..., None]                # B,H,L,1
        vb = rnd(v[:, s:e].permute(0, 2, 1, 3) * bc)                 # wy_fast.py:67
        kb = rnd(k[:, s:e].permute(0, 2, 1, 3) * bc * gc[:, s:e].permute(0, 2, 1)[..., None].exp())  # wy_fast.py:77-79
        u[:, s:e] = rnd(Ai @ vb).permute(0, 2, 1, 3)                 # wy_fast.py:68-69
        w[:, s:e] = rnd(Ai @ kb).permute(0, 2, 1, 3)                 # wy_fast.py:80-81
    # inter-chunk state pass, chunk_delta_h.py:128-211
    h = torch.zeros(B, H, K, V, dtype=dt)
    if initial_state is not None:
        h = initial_state.to(dt).clone()
    hs = []
    v_new = torch.zeros(B, T, H, V, dtype=dt)
    for s, e in chunks:
        hb = rnd(h)                                                  # snapshot stored in k.dtype (:129-140)
        hs.append(hb)
        wc = w[:, s:e].permute(0, 2, 1, 3)
        vn = u[:, s:e].permute(0, 2, 1, 3) - wc @ hb                 # :142-159
        v_new[:, s:e] = rnd(vn).permute(0, 2, 1, 3)                  # :161-163
        gcc = gc[:, s:e].permute(0, 2, 1)                            # B,H,L
        glast = gcc[..., -1]
        vg = rnd(vn * (glast[..., None] - gcc).exp()[..., None])     # :165-171, cast at :196
        h = h * glast.exp()[..., None, None]                         # :172-178
        kc = k[:, s:e].permute(0, 2, 1, 3)
        h = h + kc.transpose(-1, -2) @ vg                            # :198-210
    # output, chunk_o.py:85-126
    o = torch.zeros(B, T, H, V, dtype=dt)
    for (s, e), hb in zip(chunks, hs):
        qc = q[:, s:e].permute(0, 2, 1, 3)
        kc = k[:, s:e].permute(0, 2, 1, 3)
        gcc = gc[:, s:e].permute(0, 2, 1)
        L = e - s
        oi = (qc @ hb) * gcc.exp()[..., None]
        mask = torch.tril(torch.ones(L, L, dtype=torch.bool))
        diff = (gcc[..., :, None] - gcc[..., None, :]).masked_fill(~mask, 0.0)
        Aqk = ((qc @ kc.transpose(-1, -2)) * diff.exp()).masked_fill(~mask, 0.0)
        vn = v_new[:, s:e].permute(0, 2, 1, 3)
        oc = oi * scale + (rnd(Aqk) @ vn) * scale
        o[:, s:e] = rnd(oc).permute(0, 2, 1, 3)
    fs = h if output_final_state else None
    if return_intermediates:
        return o, fs, dict(gc=gc, Ai=Ais, w=w, u=u, v_new=v_new, h=hs)
    return o, fs


def gdn_chunk_varlen(q, k, v, g, beta, cu_seqlens, scale=None, initial_state=None,
                     output_final_state=True, use_qk_l2norm=False, emulate_bf16=False):
    """Variable-length form: B must be 1; each segment of ``cu_seqlens`` is an
    independent sequence with its own state (``chunk.py:298-308`` checks,
    ``chunk_delta_h.py:98-103`` per-sequence offsets)."""
    assert q.shape[0] == 1
    N = len(cu_seqlens) - 1
    outs, states = [], []
    for n in range(N):
        s, e = int(cu_seqlens[n]), int(cu_seqlens[n + 1])
        h0 = None if initial_state is None else initial_state[n:n + 1]
        o, st = gdn_chunk(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e], beta[:, s:e], scale, h0,
                          True, use_qk_l2norm, emulate_bf16)
        outs.append(o)
        states.append(st)
    o = torch.cat(outs, 1)
    return o, (torch.cat(states, 0) if output_final_state else None)
