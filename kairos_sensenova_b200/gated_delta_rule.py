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
reference's Triton kernels use for bf16 activations.  Inputs given in another
float dtype are converted to bf16 first.  Only the forward exists: calling it
with grad-requiring inputs under autograd raises ``NotImplementedError``.
"""
from __future__ import annotations

import ctypes
import warnings

import torch

from . import _lib

BT = 64


def _ptr(t):
    return None if t is None else t.data_ptr()


def prepare_chunk_indices(cu_seqlens: torch.Tensor, chunk_size: int = BT):
    """(seq, chunk) pairs and per-sequence chunk offsets for variable-length input
    (the same tables as ``fla/ops/utils/index.py`` ``prepare_chunk_indices`` /
    ``prepare_chunk_offsets``), built on the host."""
    lens = (cu_seqlens[1:] - cu_seqlens[:-1]).tolist()
    pairs, offs = [], [0]
    for n, ln in enumerate(lens):
        nt = (int(ln) + chunk_size - 1) // chunk_size
        pairs.extend((n, i) for i in range(nt))
        offs.append(offs[-1] + nt)
    return pairs, offs


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
                    cu_seqlens, use_qk_l2norm_in_kernel)


def _forward(q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, l2norm):
    dev = q.device
    if dev.type != 'cuda':
        raise RuntimeError('chunk_gated_delta_rule: inputs must be CUDA tensors (no CPU path)')
    B, T, H, K = q.shape
    V = v.shape[-1]
    assert K <= 256, "current kernel does not support head dimension larger than 256."
    if k.shape != q.shape or v.shape[:3] != q.shape[:3] or g.shape != q.shape[:3] or beta.shape != q.shape[:3]:
        raise ValueError(f'chunk_gated_delta_rule: inconsistent shapes q{tuple(q.shape)} k{tuple(k.shape)} '
                         f'v{tuple(v.shape)} g{tuple(g.shape)} beta{tuple(beta.shape)}')
    out_dtype = q.dtype
    with torch.cuda.device(dev):
        bf = torch.bfloat16
        qc, kc, vc = (x.to(bf).contiguous() for x in (q, k, v))
        gc = g.to(torch.float32).contiguous()
        bc = beta.to(bf).contiguous()
        if cu_seqlens is not None:
            pairs, offs = prepare_chunk_indices(cu_seqlens.cpu())
            N = len(offs) - 1
            nchunks = len(pairs)
            cu32 = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
            ci = torch.tensor(pairs if pairs else [[0, 0]], dtype=torch.int32).reshape(-1, 2).to(dev)
            co = torch.tensor(offs, dtype=torch.int32).to(dev)
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
        # kernel launches of the last call (launch accounting for benchmarks)
        chunk_gated_delta_rule.launches = L.kb200_gdn_launch_count(ctypes.byref(a))
    return o.to(out_dtype), ht
