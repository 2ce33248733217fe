"""FP8 attention module with the reference's ``AttentionModule`` interface.

``AttentionModule(num_heads).forward(q, k, v, attn_mask=None, window_size=(-1, -1))``
with q, k, v ``[B, S, N*D]`` bf16 returns ``[B, S, N*D]`` bf16
(``kairos/modules/dits/kairos_dit.py:362-373``).  The core is computed by the
sm_100a kernels behind ``kb200_attn_fp8_fwd``: per-(batch, head) amax scaling
of q/k to e4m3, non-causal softmax(q k^T / sqrt(D)) v with fp32 softmax and
accumulation; the P.V half runs on bf16 probabilities and the bf16 V (with P
and V in e4m3 too, the cosine similarity to the bf16 reference would sit near
0.9986 on N(0,1) data, below the 0.999 contract; this way it is ~0.9992).  Like the reference's
quantised backends (``SageAttention3Module``, ``kairos_dit.py:398-420``) it
raises ``NotImplementedError`` for an ``attn_mask``.  A sliding ``window_size``
(left, right) restricts query i to keys i - left .. i + right, as the reference's
flash-attention call does for ``SelfAttention`` (``kairos_dit.py:423-507``; its
dilation is a rearrangement before this call); key tiles outside every window of a
256-query block are skipped.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib


def attention_fp8(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, num_heads: int,
                  softmax_scale: float | None = None,
                  events=None, check: bool = False, window_size=(-1, -1)) -> torch.Tensor:
    """q, k, v: [B, S, H*D] (bf16; other float dtypes are converted) -> [B, S, H*D] bf16.

    ``events``: optional (start, end) CUDA events recorded on the launch stream
    around the attention kernel alone (after quantisation).  ``window_size``:
    (left, right) sliding window as in flash-attention (query i sees keys
    i - left .. i + right; -1 = unbounded)."""
    if q.device.type != 'cuda':
        raise RuntimeError('attention_fp8: inputs must be CUDA tensors (no CPU path)')
    if q.dim() != 3 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f'attention_fp8: q/k/v must share shape [B,S,H*D], got {tuple(q.shape)}, '
                         f'{tuple(k.shape)}, {tuple(v.shape)}')
    B, S, HD = q.shape
    if HD % num_heads:
        raise ValueError(f'attention_fp8: hidden {HD} not divisible by num_heads {num_heads}')
    D = HD // num_heads
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    dev = q.device
    with torch.cuda.device(dev):
        qc, kc, vc = (x.to(torch.bfloat16) for x in (q, k, v))
        ld = qc.stride(1)
        # strided row views (e.g. column slices of one projection) are read in place
        if not all(t.stride(2) == 1 and t.stride(1) == ld and (B == 1 or t.stride(0) == S * ld)
                   and t.data_ptr() % 16 == 0 for t in (qc, kc, vc)) or ld % 8:
            qc, kc, vc = (t.contiguous() for t in (qc, kc, vc))
            ld = HD
        o = torch.empty(B, S, HD, device=dev, dtype=torch.bfloat16)
        L = _lib.lib()
        nbytes = L.kb200_attn_fp8_workspace_size(B, S, num_heads, D)
        if nbytes == 0:
            raise ValueError(f'attention_fp8: unsupported shape B={B} S={S} H={num_heads} D={D} (D must be 128)')
        ws = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        stream = torch.cuda.current_stream(dev).cuda_stream
        args = (qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), B, S, num_heads, D, ld,
                float(softmax_scale), ws.data_ptr(), nbytes, stream)
        wl, wr = (int(x) for x in window_size)
        windowed = wl >= 0 or wr >= 0
        if events is None:
            if windowed:
                _lib.check(L.kb200_attn_fp8_fwd_window(*args, wl, wr), 'attention_fp8')
            else:
                _lib.check(L.kb200_attn_fp8_fwd(*args), 'attention_fp8')
        else:
            _lib.check(L.kb200_attn_fp8_quantize(*args), 'attention_fp8 quantize')
            events[0].record()
            if windowed:
                _lib.check(L.kb200_attn_fp8_attend_window(*args, wl, wr), 'attention_fp8 attend')
            else:
                _lib.check(L.kb200_attn_fp8_attend(*args), 'attention_fp8 attend')
            events[1].record()
        if check:   # synchronises; raises if a bounded device wait gave up
            _lib.check(L.kb200_attn_fp8_status(ws.data_ptr(), B, S, num_heads, stream),
                       'attention_fp8')
    return o


class AttentionModule(nn.Module):
    """Drop-in for ``AttentionModule`` / ``SageAttention3Module`` (``kairos_dit.py:362-420``)."""

    def __init__(self, num_heads):
        super().__init__()
        self.num_heads = num_heads

    def forward(self, q, k, v, attn_mask=None, window_size=(-1, -1)):
        if attn_mask is not None:
            raise NotImplementedError('FP8 attention path does not support arbitrary attn_mask')
        return attention_fp8(q, k, v, self.num_heads, window_size=window_size)


FP8AttentionModule = AttentionModule
