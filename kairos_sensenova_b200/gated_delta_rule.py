"""Drop-in ``chunk_gated_delta_rule`` backed by the sm_100a kernels.

Same signature, argument meaning, defaults and errors as the reference op
``chunk_gated_delta_rule`` (``kairos/third_party/fla/ops/gated_delta_rule/chunk.py:216-323``):

* q, k ``[B,T,H,K]``, v ``[B,T,H,V]``, g ``[B,T,H]`` (log-space decay),
  beta ``[B,T,H]``; ``scale`` defaults to ``K ** -0.5`` (``chunk.py:309-310``);
* ``initial_state [N,H,K,V]``; with ``cu_seqlens`` the batch must be 1 and N
  must equal ``len(cu_seqlens)-1``, otherwise ``ValueError`` (``chunk.py:298-308``);
* returns ``(o, final_state)``: o in ``q.dtype``, final_state fp32 ``[N,H,K,V]``
  or ``None`` when ``output_final_state`` is False;
* inputs are made contiguous and the launch runs on the current CUDA stream
  of the inputs' device (``input_guard``, ``fla/utils.py:135-164``).

Arithmetic: bf16 operands (q, k, v, beta, w, u, state snapshots) with fp32
accumulation, fp32 gates and an fp32 running state -- the precision the
reference's Triton kernels use for bf16 activations.  q, k and v must be bf16:
other dtypes raise ``ValueError`` (the reference would compute fp32 inputs in
fp32; this op has no fp32 path, and silently rounding them would change the
results).  g may be any float dtype (it is used in fp32, like the reference);
beta is used in bf16 (fp32 beta is rounded, a 2^-9 relative change).  Only the
forward exists: calling it with grad-requiring inputs under autograd raises
``NotImplementedError``.  ``check=True`` (an extra keyword; the reference's
``**kwargs`` ignores it) synchronises after the launch and raises
``RuntimeError`` if a bounded device-side wait gave up.

Variable-length input (``cu_seqlens``) needs no host synchronisation: the
(sequence, chunk) table is built on the device for the upper bound
``ceil(T/64) + N`` of the chunk count, with unused rows marked empty.
"""
from __future__ import annotations

import ctypes
import warnings

import torch

from . import _lib

BT = 64


def _ptr(t):
    return None if t is None else t.data_ptr()


def prepare_chunk_indices(cu_seqlens: torch.Tensor, total_tokens: int, chunk_size: int = BT):
    """(sequence, chunk) rows and per-sequence chunk offsets for variable-length
    input (the tables of ``fla/ops/utils/index.py`` ``prepare_chunk_indices`` /
    ``prepare_chunk_offsets``), built with device ops only (no host sync).

    Returns ``(indices [M, 2] int32, offsets [N+1] int32, M)`` with
    ``M = ceil(total_tokens / chunk_size) + N`` -- an upper bound of the chunk
    count known from shapes alone; rows past the real chunk count hold
    sequence -1 and are skipped by the kernels."""
    N = cu_seqlens.shape[0] - 1
    M = (total_tokens + chunk_size - 1) // chunk_size + N
    cu = cu_seqlens.to(torch.int64)
    nt = (cu[1:] - cu[:-1] + chunk_size - 1) // chunk_size
    offs = torch.cat([nt.new_zeros(1), torch.cumsum(nt, 0)])
    c = torch.arange(M, device=cu.device, dtype=torch.int64)
    n = torch.searchsorted(offs[1:].contiguous(), c, right=True)
    valid = n < N
    nc = n.clamp(max=max(N - 1, 0))
    it = c - offs[nc]
    idx = torch.stack([torch.where(valid, nc, torch.full_like(nc, -1)), torch.where(valid, it, 0)], 1)
    return idx.to(torch.int32).contiguous(), offs.to(torch.int32).contiguous(), M


@torch.compiler.disable
def chunk_gated_delta_rule(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    scale: float = None,
    initial_state: torch.Tensor = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    cu_seqlens: torch.LongTensor | None = None,
    **kwargs,
):
    if 'head_first' in kwargs:
        warnings.warn(
            "head_first is deprecated and will be removed in a future version. "
            "Please use head_first=False for now instead.",
        )
    if cu_seqlens is not None:
        if q.shape[0] != 1:
            raise ValueError(
                f"The batch size is expected to be 1 rather than {q.shape[0]} when using `cu_seqlens`."
                f"Please flatten variable-length inputs before processing.",
            )
        if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
            raise ValueError(
                f"The number of initial states is expected to be equal to the number of input sequences, "
                f"i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}.",
            )
    if scale is None:
        scale = k.shape[-1] ** -0.5
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (q, k, v, g, beta, initial_state)):
        raise NotImplementedError('kairos_sensenova_b200.chunk_gated_delta_rule is forward-only')
    return _forward(q, k, v, g, beta, float(scale), initial_state, output_final_state,
                    cu_seqlens, use_qk_l2norm_in_kernel, bool(kwargs.get('check', False)))


def _forward(q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, l2norm, check=False):
    dev = q.device
    if dev.type != 'cuda':
        raise RuntimeError('chunk_gated_delta_rule: inputs must be CUDA tensors (no CPU path)')
    B, T, H, K = q.shape
    V = v.shape[-1]
    assert K <= 256, "current kernel does not support head dimension larger than 256."
    if k.shape != q.shape or v.shape[:3] != q.shape[:3] or g.shape != q.shape[:3] or beta.shape != q.shape[:3]:
        raise ValueError(f'chunk_gated_delta_rule: inconsistent shapes q{tuple(q.shape)} k{tuple(k.shape)} '
                         f'v{tuple(v.shape)} g{tuple(g.shape)} beta{tuple(beta.shape)}')
    bf = torch.bfloat16
    if q.dtype != bf or k.dtype != bf or v.dtype != bf:
        raise ValueError(f'chunk_gated_delta_rule: q, k, v must be bfloat16 (this op computes in bf16 with fp32 '
                         f'accumulation and has no fp32 path), got {q.dtype}, {k.dtype}, {v.dtype}')
    with torch.cuda.device(dev):
        qc, kc, vc = (x.contiguous() for x in (q, k, v))
        gc = g.to(torch.float32).contiguous()
        bc = beta.to(bf).contiguous()
        if cu_seqlens is not None:
            cu_dev = cu_seqlens.to(device=dev)
            ci, co, nchunks = prepare_chunk_indices(cu_dev, B * T)
            N = cu_seqlens.shape[0] - 1
            cu32 = cu_dev.to(torch.int32).contiguous()
        else:
            N = B
            nchunks = B * ((T + BT - 1) // BT)
            cu32 = ci = co = None
        h0 = None
        if initial_state is not None:
            if tuple(initial_state.shape) != (N, H, K, V):
                raise ValueError(f'initial_state must be [{N},{H},{K},{V}], got {tuple(initial_state.shape)}')
            h0 = initial_state.to(torch.float32).contiguous()
        o = torch.empty(B, T, H, V, device=dev, dtype=bf)
        ht = torch.empty(N, H, K, V, device=dev, dtype=torch.float32) if output_final_state else None
        a = _lib.GdnArgs(
            q=_ptr(qc), k=_ptr(kc), v=_ptr(vc), g=_ptr(gc), beta=_ptr(bc), initial_state=_ptr(h0),
            o=_ptr(o), final_state=_ptr(ht), cu_seqlens=_ptr(cu32), chunk_indices=_ptr(ci),
            chunk_offsets=_ptr(co), B=B, T=T, H=H, K=K, V=V, N=N, num_chunks=nchunks,
            scale=scale, use_qk_l2norm=int(bool(l2norm)))
        L = _lib.lib()
        nbytes = L.kb200_gdn_workspace_size(ctypes.byref(a))
        if nbytes == 0:
            _lib.check(1, 'chunk_gated_delta_rule')
        ws = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(L.kb200_gdn_chunk_fwd(ctypes.byref(a), ws.data_ptr(), nbytes, stream),
                   'chunk_gated_delta_rule')
        if check:   # synchronises; raises if a bounded device-side wait gave up
            _lib.check(L.kb200_gdn_status(ws.data_ptr(), stream), 'chunk_gated_delta_rule')
        # kernel launches of the last call (launch accounting for benchmarks)
        chunk_gated_delta_rule.launches = L.kb200_gdn_launch_count(ctypes.byref(a))
    return o, ht
