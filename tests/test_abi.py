"""C-ABI library: loads, exports every symbol include/kb200.h declares, and
rejects bad arguments without touching a GPU (the validators run on the host)."""
import ctypes
import re
from pathlib import Path

import pytest

from kairos_sensenova_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / 'include' / 'kb200.h'


def declared_symbols():
    return sorted(set(re.findall(r'\b(kb200_[a-z0-9_]+)\s*\(', HEADER.read_text())))


def test_library_loads_and_exports_all_declared_symbols():
    L = _lib.lib()
    syms = declared_symbols()
    assert 'kb200_gdn_chunk_fwd' in syms
    for s in syms:
        assert hasattr(L, s), s
        assert s in _lib.SIGNATURES, f'{s} has no ctypes signature'


def test_abi_version():
    assert _lib.lib().kb200_abi_version() == 2


def _args(**kw):
    base = dict(q=16, k=16, v=16, g=16, beta=16, o=16, B=1, T=100, H=2, K=128, V=128, N=1,
                num_chunks=2, scale=1.0, use_qk_l2norm=1)
    base.update(kw)
    return _lib.GdnArgs(**base)


def test_gdn_workspace_size_and_validation():
    L = _lib.lib()
    a = _args()
    n = L.kb200_gdn_workspace_size(ctypes.byref(a))
    # K = 128 (tcgen05 path): per (chunk, head) the W (16 KB), U^T (V*128 B), Aqk (8 KB)
    # and gate-factor (528 B) blobs, plus the normalised q, k copies
    TT, H, K, V, C = 100, 2, 128, 128, 2
    assert n >= C * H * (16384 + V * 128 + 8192 + 528) + 2 * TT * H * K * 2
    # K = 256 (mma.sync path): gc + w + u + v_new + h snapshots + normalised q,k
    n256 = L.kb200_gdn_workspace_size(ctypes.byref(_args(K=256)))
    assert n256 >= TT * H * (4 + 2 * 256 * 2 + 2 * 256 + 2 * V * 2) + 2 * H * 256 * V * 2
    for bad in (dict(K=96), dict(V=64), dict(num_chunks=3), dict(B=0)):
        assert L.kb200_gdn_workspace_size(ctypes.byref(_args(**bad))) == 0
    rc = L.kb200_gdn_chunk_fwd(ctypes.byref(_args(K=96)), None, 0, None)
    assert rc == 1 and b'unsupported head dims' in L.kb200_last_error()
    rc = L.kb200_gdn_chunk_fwd(ctypes.byref(_args(q=8)), None, 0, None)
    assert rc == 2
    rc = L.kb200_gdn_chunk_fwd(ctypes.byref(_args()), None, 0, None)
    assert rc == 3 and b'workspace' in L.kb200_last_error()


def test_python_op_rejects_cpu_and_grad():
    import torch
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    q = torch.zeros(1, 4, 1, 128)
    with pytest.raises(RuntimeError, match='CUDA'):
        chunk_gated_delta_rule(q, q, q, q[..., 0], q[..., 0])
    with pytest.raises(ValueError, match='batch size'):
        chunk_gated_delta_rule(torch.zeros(2, 4, 1, 128), q, q, q[..., 0], q[..., 0],
                               cu_seqlens=torch.tensor([0, 4]))
    qg = q.clone().requires_grad_()
    with pytest.raises(NotImplementedError):
        chunk_gated_delta_rule(qg, q, q, q[..., 0], q[..., 0])


def test_gdn_state_plan_launch_count(monkeypatch):
    """The state-pass plan is host logic.  K = 128 (tcgen05 kernels): one prep launch,
    then one state launch, or three (segment-local pass, combine, final pass) when
    one CTA per (sequence x head, V slice) leaves SMs idle and every segment keeps
    >= 16 chunks; no segments for short or variable-length input.  K = 256 (mma.sync
    kernels): 3 launches, 5 with segments.  (Without a GPU the plan assumes B200's
    148 SMs.)"""
    L = _lib.lib()
    monkeypatch.delenv('KB200_GDN_SEGMENTS', raising=False)
    monkeypatch.delenv('KB200_GDN_STATE_BV', raising=False)
    cnt = lambda **kw: L.kb200_gdn_launch_count(ctypes.byref(_args(**kw)))  # noqa: E731
    nt = lambda T: (T + 63) // 64  # noqa: E731
    assert cnt(T=32760, H=24, num_chunks=nt(32760)) == 4
    assert cnt(T=32760, H=3, num_chunks=nt(32760)) == 4
    assert cnt(T=32760, H=160, num_chunks=nt(32760)) == 2     # the heads alone fill the SMs
    assert cnt(T=200, H=3, num_chunks=nt(200)) == 2
    assert cnt(T=0, H=3, num_chunks=0) == 1           # no chunks: the state pass only (h0 -> ht)
    assert cnt(K=96) == -1
    assert cnt(K=256, V=256, T=32760, H=3, num_chunks=nt(32760)) == 5
    seg = L.kb200_gdn_workspace_size(ctypes.byref(_args(T=32760, H=3, num_chunks=nt(32760))))
    monkeypatch.setenv('KB200_GDN_SEGMENTS', '1')
    assert cnt(T=32760, H=3, num_chunks=nt(32760)) == 2
    one = L.kb200_gdn_workspace_size(ctypes.byref(_args(T=32760, H=3, num_chunks=nt(32760))))
    # segments add the local end states, transitions and start states (fp32)
    assert seg - one >= 3 * 6 * (128 * 128 * 4) * 3
