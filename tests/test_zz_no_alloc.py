"""The allocation-free GDN entry point, called through the C ABI.

``kb200_gdn_chunk_fwd_noalloc`` serves callers that cannot allocate device
memory while they run the operator (for example a plugin host that owns all
device memory and passes in only the inputs and outputs): its scratch is a
fixed array built into the library.  This test checks, for two calls in a
row, that it returns what the workspace-taking ``kb200_gdn_chunk_fwd``
returns on the same inputs, and that over-sized problems are refused.

It sits in a file of its own that pytest collects last.
"""
import ctypes

import pytest
import torch

from conftest import max_rel

pytestmark = pytest.mark.gpu


def _case(seed, T, H, K=128, V=128, h0=True):
    gen = torch.Generator().manual_seed(seed)
    c = lambda x, dt=torch.bfloat16: x.to('cuda', dt).contiguous()  # noqa: E731
    q, k = c(torch.randn(1, T, H, K, generator=gen)), c(torch.randn(1, T, H, K, generator=gen))
    v = c(torch.randn(1, T, H, V, generator=gen))
    g = c(-torch.rand(1, T, H, generator=gen), torch.float32)
    beta = c(torch.rand(1, T, H, generator=gen))
    init = c(torch.randn(1, H, K, V, generator=gen) * 0.1, torch.float32) if h0 else None
    return q, k, v, g, beta, init


def _args(q, k, v, g, beta, init, o, ht):
    from kairos_sensenova_b200 import _lib
    B, T, H, K = q.shape
    V = v.shape[-1]
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    return _lib.GdnArgs(q=p(q), k=p(k), v=p(v), g=p(g), beta=p(beta), initial_state=p(init), o=p(o),
                        final_state=p(ht), B=B, T=T, H=H, K=K, V=V, N=B, num_chunks=B * ((T + 63) // 64),
                        scale=K ** -0.5, use_qk_l2norm=1)


def _run_with_workspace(L, inputs):
    q, v = inputs[0], inputs[2]
    o = torch.empty(*q.shape[:3], v.shape[-1], device='cuda', dtype=torch.bfloat16)
    ht = torch.empty(1, q.shape[2], q.shape[3], v.shape[-1], device='cuda', dtype=torch.float32)
    a = _args(*inputs, o, ht)
    n = L.kb200_gdn_workspace_size(ctypes.byref(a))
    ws = torch.empty(n, device='cuda', dtype=torch.uint8)
    assert L.kb200_gdn_chunk_fwd(ctypes.byref(a), ws.data_ptr(), n,
                                 torch.cuda.current_stream().cuda_stream) == 0
    return o, ht


def _run_noalloc(L, inputs):
    q, v = inputs[0], inputs[2]
    o = torch.empty(*q.shape[:3], v.shape[-1], device='cuda', dtype=torch.bfloat16)
    ht = torch.empty(1, q.shape[2], q.shape[3], v.shape[-1], device='cuda', dtype=torch.float32)
    a = _args(*inputs, o, ht)
    rc = L.kb200_gdn_chunk_fwd_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, L.kb200_last_error()
    return o, ht


def test_noalloc_matches_workspace_entry_point_twice():
    from kairos_sensenova_b200 import _lib
    L = _lib.lib()
    torch.cuda.set_device(0)
    # two different problems back to back: the second call reuses the array
    # that still holds the first call's intermediates
    for seed, T, H in ((1, 1000, 4), (2, 333, 3)):
        inputs = _case(seed, T, H)
        o_ref, s_ref = _run_with_workspace(L, inputs)
        o, s = _run_noalloc(L, inputs)
        torch.cuda.synchronize()
        assert max_rel(o, o_ref) <= 2e-2 and max_rel(s, s_ref) <= 1e-2
        assert torch.equal(o, o_ref) and torch.equal(s, s_ref)   # same kernels, same order


def test_noalloc_rejects_oversized_problem():
    from kairos_sensenova_b200 import _lib
    L = _lib.lib()
    cap = L.kb200_gdn_noalloc_scratch_bytes()
    assert cap == 64 << 20
    T, H = 65536, 4                                    # needs far more than 64 MiB
    a = _lib.GdnArgs(q=16, k=16, v=16, g=16, beta=16, o=16, B=1, T=T, H=H, K=128, V=128, N=1,
                     num_chunks=(T + 63) // 64, scale=1.0, use_qk_l2norm=1)
    assert L.kb200_gdn_workspace_size(ctypes.byref(a)) > cap
    rc = L.kb200_gdn_chunk_fwd_noalloc(ctypes.byref(a), None)
    assert rc == 3 and b'built-in array' in L.kb200_last_error()
