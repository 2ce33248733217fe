"""Python entry points of the prologue / epilogue fusion kernels.

* :func:`gdn_prologue` -- ShortConvolution(q,k,v)+SiLU and the beta/g gates of
  ``GatedDeltaNet.forward`` (``kairos/third_party/fla/layers/gated_deltanet.py:238-271``)
  in one launch.
* :func:`rms_norm_gated` -- ``FusedRMSNormGated`` (swish gate) forward
  (``fla/modules/fused_norm_gate.py:1024-1085``).
* :func:`rmsnorm_rope` -- the attention prologue: full-dim RMSNorm (+ 3-D RoPE).
* :func:`residual_ln_mod` -- the DiT block's residual add + LayerNorm +
  modulation sites (``kairos_dit.py:306-309, 873-874, 929-957``).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _rows(x, C):
    """Validate a [*, C] bf16 row view with unit column stride; return (tensor, row stride)."""
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    x2 = x.reshape(-1, C) if x.is_contiguous() else x
    if x2.dim() != 2 or x2.stride(-1) != 1:
        x2 = x2.contiguous().reshape(-1, C)
    return x2, x2.stride(0)


def gdn_prologue(xq, xk, xv, a, b, wq, wk, wv, A_log, dt_bias, num_heads, B, T,
                 bq=None, bk=None, bv=None, allow_neg_eigval=False, conv_cache=None):
    """xq/xk/xv: bf16 [B*T, C] row views (may be column slices of one fused
    projection), a/b: bf16 [B*T, H] row views, conv weights [C, W].
    ``conv_cache``: optional ``(cq, ck, cv)`` conv states ``[B, C, W]`` of the
    preceding piece of each sequence (ShortConvolution's ``cache``,
    ``fla/modules/convolution.py:771-798``); their last W-1 columns are the
    inputs just before token 0.  They are read, not updated.
    Returns q, k [B,T,H,Cqk/H], v [B,T,H,Cv/H] bf16, g fp32 [B,T,H], beta bf16 [B,T,H]."""
    dev = xq.device
    if dev.type != 'cuda':
        raise RuntimeError('gdn_prologue: CUDA tensors required (no CPU path)')
    Cqk, Cv = wq.shape[0], wv.shape[0]
    W = wq.shape[-1]
    H = num_heads
    xq, ldq = _rows(xq, Cqk)
    xk, ldk = _rows(xk, Cqk)
    xv, ldv = _rows(xv, Cv)
    a, lda = _rows(a, H)
    b, ldb = _rows(b, H)
    f32 = lambda t: None if t is None else t.to(device=dev, dtype=torch.float32).reshape(t.shape[0], -1).contiguous()  # noqa: E731
    wq, wk, wv = f32(wq), f32(wk), f32(wv)
    bq, bk, bv = (None if t is None else t.to(dev, torch.float32).contiguous() for t in (bq, bk, bv))
    A = A_log.to(dev, torch.float32).contiguous()
    dtb = dt_bias.to(dev, torch.float32).contiguous()
    q = torch.empty(B, T, H, Cqk // H, device=dev, dtype=torch.bfloat16)
    k = torch.empty_like(q)
    v = torch.empty(B, T, H, Cv // H, device=dev, dtype=torch.bfloat16)
    g = torch.empty(B, T, H, device=dev, dtype=torch.float32)
    beta = torch.empty(B, T, H, device=dev, dtype=torch.bfloat16)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    caches = [None, None, None]
    if conv_cache is not None:
        for i, (c, C) in enumerate(zip(conv_cache, (Cqk, Cqk, Cv))):
            if c is None:
                continue
            if tuple(c.shape) != (B, C, W):
                raise ValueError(f'gdn_prologue: conv state must be [{B},{C},{W}], got {tuple(c.shape)}')
            caches[i] = c.to(device=dev, dtype=torch.bfloat16).contiguous()
    args = _lib.GdnPrologueArgs(
        xq=p(xq), xk=p(xk), xv=p(xv), ldq=ldq, ldk=ldk, ldv=ldv, wq=p(wq), wk=p(wk), wv=p(wv),
        bq=p(bq), bk=p(bk), bv=p(bv), q=p(q), k=p(k), v=p(v), a=p(a), b=p(b), lda=lda, ldb=ldb,
        A_log=p(A), dt_bias=p(dtb), g=p(g), beta=p(beta), B=B, T=T, H=H, Cqk=Cqk, Cv=Cv, W=W,
        allow_neg_eigval=int(bool(allow_neg_eigval)),
        cache_q=p(caches[0]), cache_k=p(caches[1]), cache_v=p(caches[2]))
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().kb200_gdn_prologue(ctypes.byref(args), _stream(dev)), 'gdn_prologue')
    return q, k, v, g, beta


def rms_norm_gated(x: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5):
    """x: [..., H, D] bf16; gate: same logical shape (token rows may be strided);
    weight [D].  Returns bf16 like x."""
    dev = x.device
    if dev.type != 'cuda':
        raise RuntimeError('rms_norm_gated: CUDA tensors required (no CPU path)')
    D = x.shape[-1]
    H = x.shape[-2] if x.dim() >= 2 else 1
    xc = x.to(torch.bfloat16).contiguous()
    g2 = gate.to(torch.bfloat16)
    g2 = g2.reshape(-1, H * D) if g2.is_contiguous() else g2.contiguous().reshape(-1, H * D)
    w = weight.to(dev, torch.float32).contiguous()
    y = torch.empty_like(xc)
    rows = xc.numel() // D
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().kb200_rmsnorm_gated(xc.data_ptr(), g2.data_ptr(), w.data_ptr(), y.data_ptr(),
                                                   rows, H, D, g2.stride(0), float(eps), _stream(dev)),
                   'rms_norm_gated')
    return y


def freqs_cis_3d(head_dim: int, f: int, h: int, w: int, theta: float = 10000.0) -> torch.Tensor:
    """Per-token complex RoPE factors [f*h*w, head_dim/2] for a (frame, height,
    width) latent grid: the frame axis gets head_dim - 2*(head_dim//3) channels,
    height and width head_dim//3 each (``precompute_freqs_cis_3d``,
    ``kairos_dit.py:312-315``; per-token layout as ``KairosDiT.forward``,
    ``kairos_dit.py:1217-1221``)."""
    def one(dim, end):
        fr = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].double() / dim))
        return torch.polar(torch.ones(end, dim // 2, dtype=torch.float64),
                           torch.outer(torch.arange(end, dtype=torch.float64), fr))
    ff = one(head_dim - 2 * (head_dim // 3), f)
    fh = one(head_dim // 3, h)
    fw = one(head_dim // 3, w)
    return torch.cat([ff.view(f, 1, 1, -1).expand(f, h, w, -1), fh.view(1, h, 1, -1).expand(f, h, w, -1),
                      fw.view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(f * h * w, -1)


def rope_table(freqs: torch.Tensor, device) -> torch.Tensor:
    """Complex factors [S, D/2] (or [S, 1, D/2]) -> interleaved (cos, sin) fp32 [S, D/2, 2]."""
    fr = freqs.reshape(freqs.shape[0], -1)
    return torch.stack([fr.real, fr.imag], dim=-1).to(device=device, dtype=torch.float32).contiguous()


def rmsnorm_rope(x: torch.Tensor, weight, cos_sin: torch.Tensor, head_dim: int, eps: float = 1e-6,
                 out: torch.Tensor | None = None, rows: int | None = None, dim: int | None = None,
                 ld: int | None = None, heads_per_block: int | None = None, block_stride: int = 0):
    """``RoPE(RMSNorm(x) * weight)`` per token row (``SelfAttention.forward``,
    ``kairos_dit.py:452-456``).  ``x``: [..., dim] bf16 (rows = all leading
    elements) or, with ``rows/dim/ld/heads_per_block/block_stride``, a
    destination-grouped projection view; ``out`` defaults to a new tensor
    (pass ``out=x`` to work in place).  ``cos_sin=None``: plain RMSNorm."""
    dev = x.device
    if dev.type != 'cuda':
        raise RuntimeError('rmsnorm_rope: CUDA tensors required (no CPU path)')
    if dim is None:
        xc = x.to(torch.bfloat16).contiguous()
        dim = xc.shape[-1]
        rows = xc.numel() // dim
        ld = dim
        heads_per_block = dim // head_dim
        x = xc
    if out is None:
        out = torch.empty_like(x)
    w = None if weight is None else weight.to(dev, torch.float32).contiguous()
    cs = None if cos_sin is None else cos_sin.to(dev, torch.float32).contiguous()
    if cs is not None and cs.numel() < rows * head_dim:
        raise ValueError('rmsnorm_rope: cos/sin table smaller than rows x head_dim/2 x 2')
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().kb200_rmsnorm_rope(x.data_ptr(), out.data_ptr(), rows, dim, head_dim, ld,
                                                  heads_per_block, block_stride,
                                                  None if w is None else w.data_ptr(),
                                                  None if cs is None else cs.data_ptr(),
                                                  float(eps), _stream(dev)),
                   'rmsnorm_rope')
    return out


def _vec(t, dev):
    return None if t is None else t.to(device=dev, dtype=torch.float32).contiguous()


def residual_ln_mod(x: torch.Tensor, r, gate, mul, add, mul_plus_one: bool = True, eps: float = 1e-6,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """``x <- x + gate * r`` in place (when ``r`` is given; ``gate`` None = 1), then
    ``out = LN(x) * m + add`` with ``m = 1 + mul`` (``mul_plus_one``) or ``mul``
    (None: 1; ``add`` None: 0).  x: [rows, dim] bf16 contiguous; r: [rows, dim]
    bf16 rows with unit column stride; gate/mul/add: [dim] vectors."""
    dev = x.device
    if dev.type != 'cuda':
        raise RuntimeError('residual_ln_mod: CUDA tensors required (no CPU path)')
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.dim() != 2:
        raise ValueError('residual_ln_mod: x must be a contiguous 2-D bf16 tensor (updated in place)')
    rows, dim = x.shape
    ldr = 0
    if r is not None:
        if r.shape[-1] != dim or r.numel() != rows * dim:
            raise ValueError(f'residual_ln_mod: r must hold [{rows}, {dim}], got {tuple(r.shape)}')
        r, ldr = _rows(r, dim)
    for name, v in (('gate', gate), ('mul', mul), ('add', add)):
        if v is not None and v.numel() != dim:
            raise ValueError(f'residual_ln_mod: {name} must have {dim} elements, got {v.numel()}')
    if out is None:
        out = torch.empty_like(x)
    g, m, a = _vec(gate, dev), _vec(mul, dev), _vec(add, dev)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().kb200_residual_ln_mod(x.data_ptr(), p(r), rows, dim, ldr, p(g), p(m), p(a),
                                                     int(bool(mul_plus_one)), float(eps), out.data_ptr(),
                                                     _stream(dev)), 'residual_ln_mod')
    return out
