"""GPU parity of the sm_100a GDN chunk forward against the reference's own
outputs (golden fixtures) and the CPU oracle.

Tolerances (from the parity contract): bf16 output max-relative error
<= 2e-2 and final state <= 1e-2 versus the reference fp32 path, with
max-relative = max|x - ref| / max|ref|.
"""
import glob

import pytest
import torch

from conftest import GOLDEN, max_rel

pytestmark = pytest.mark.gpu
O_TOL, S_TOL = 2e-2, 1e-2
CASES = sorted(glob.glob(str(GOLDEN / 'gdn_*.pt')))


def _dev(d, key, dtype):
    x = d[key]
    return None if x is None else x.to('cuda', dtype)


@pytest.mark.parametrize('path', CASES, ids=lambda p: p.rsplit('/', 1)[-1])
def test_gdn_golden(path):
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    d = torch.load(path)
    bf = torch.bfloat16
    q, k, v, beta = (_dev(d, n, bf) for n in ('q', 'k', 'v', 'beta'))
    g = _dev(d, 'g', torch.float32)
    h0 = _dev(d, 'h0', torch.float32)
    o, s = chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0, output_final_state=True,
                                  use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert o.dtype == bf and s.dtype == torch.float32
    assert max_rel(o, d['o_triton']) <= O_TOL
    assert max_rel(s, d['s_triton']) <= S_TOL
    assert max_rel(o, d['o_naive']) <= O_TOL


def test_gdn_matches_bf16_oracle_model_closely():
    """The kernel rounds where the bf16 oracle model rounds: agreement is much
    tighter than the contract tolerance."""
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    from oracle import gdn as og
    d = torch.load(GOLDEN / 'gdn_t1000.pt')
    args = [d[n].float() for n in ('q', 'k', 'v', 'g', 'beta')]
    ob, sb = og.gdn_chunk(*args, None, d['h0'], True, use_qk_l2norm=True, emulate_bf16=True)
    bf = torch.bfloat16
    o, s = chunk_gated_delta_rule(*(a.to('cuda', bf if i != 3 else torch.float32) for i, a in enumerate(args)),
                                  initial_state=d['h0'].cuda(), output_final_state=True,
                                  use_qk_l2norm_in_kernel=True)
    assert max_rel(o, ob) < 1e-2
    assert max_rel(s, sb) < 5e-3


def test_gdn_no_l2norm_and_scale():
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    from oracle import gdn as og
    gen = torch.Generator().manual_seed(5)
    B, T, H, K, V = 1, 300, 3, 128, 128
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=gen), dim=-1).bfloat16().float()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=gen), dim=-1).bfloat16().float()
    v = torch.randn(B, T, H, V, generator=gen).bfloat16().float()
    beta = torch.rand(B, T, H, generator=gen).bfloat16().float()
    g = -torch.rand(B, T, H, generator=gen)
    oref, sref = og.gdn_chunk(q, k, v, g, beta, 0.25, None, True, use_qk_l2norm=False)
    c = lambda x, dt=torch.bfloat16: x.to('cuda', dt)  # noqa: E731
    o, s = chunk_gated_delta_rule(c(q), c(k), c(v), c(g, torch.float32), c(beta), scale=0.25,
                                  output_final_state=True)
    assert max_rel(o, oref) <= O_TOL and max_rel(s, sref) <= S_TOL
    o2, s2 = chunk_gated_delta_rule(c(q), c(k), c(v), c(g, torch.float32), c(beta), scale=0.25)
    assert s2 is None and torch.equal(o, o2)   # deterministic


def test_gdn_varlen_matches_separate_calls():
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    gen = torch.Generator().manual_seed(6)
    lens = [1, 63, 64, 65, 200]
    T, H, K, V = sum(lens), 2, 128, 128
    q, k = torch.randn(1, T, H, K, generator=gen), torch.randn(1, T, H, K, generator=gen)
    v = torch.randn(1, T, H, V, generator=gen)
    beta = torch.rand(1, T, H, generator=gen)
    g = -torch.rand(1, T, H, generator=gen)
    h0 = torch.randn(len(lens), H, K, V, generator=gen) * 0.1
    c = lambda x, dt=torch.bfloat16: x.to('cuda', dt)  # noqa: E731
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device='cuda')
    o, s = chunk_gated_delta_rule(c(q), c(k), c(v), c(g, torch.float32), c(beta), initial_state=c(h0, torch.float32),
                                  output_final_state=True, use_qk_l2norm_in_kernel=True, cu_seqlens=cu)
    st = 0
    for i, ln in enumerate(lens):
        sl = slice(st, st + ln)
        oi, si = chunk_gated_delta_rule(c(q[:, sl]), c(k[:, sl]), c(v[:, sl]), c(g[:, sl], torch.float32),
                                        c(beta[:, sl]), initial_state=c(h0[i:i + 1], torch.float32),
                                        output_final_state=True, use_qk_l2norm_in_kernel=True)
        assert torch.equal(o[:, sl], oi)
        assert torch.equal(s[i:i + 1], si)
        st += ln


def test_gdn_config1_full_size_two_heads_vs_oracle():
    """BASELINE config 1 shape (T=32760, H=24, d=128) on the GPU; heads are
    independent, so two of them are checked against the fp32 oracle."""
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    from kairos_sensenova_b200.inputs import gdn_inputs
    from oracle import gdn as og
    q, k, v, g, beta = gdn_inputs(1, 32760, 24, 128, 128, seed=0, device='cuda')
    o, s = chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(s).all()
    for h in (0, 23):
        sl = lambda x: x[:, :, h:h + 1].float().cpu()  # noqa: E731
        oref, sref = og.gdn_chunk(sl(q), sl(k), sl(v), sl(g), sl(beta), None, None, True, use_qk_l2norm=True)
        assert max_rel(o[:, :, h:h + 1], oref) <= O_TOL
        assert max_rel(s[:, h:h + 1], sref) <= S_TOL


def _seg_inputs(T, H, K, V, seed, decay=0.01):
    gen = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1)
    v = torch.randn(1, T, H, V, generator=gen)
    beta = torch.sigmoid(torch.randn(1, T, H, generator=gen))
    g = -torch.nn.functional.softplus(torch.randn(1, T, H, generator=gen)) * decay
    h0 = torch.randn(1, H, K, V, generator=gen) * 0.1
    return [x.bfloat16().float() for x in (q, k, v)] + [g, beta.bfloat16().float(), h0]


@pytest.mark.parametrize('T,H,K,V', [(4000, 2, 128, 128), (2048, 1, 256, 512)])
def test_gdn_segmented_state_pass_vs_oracle(T, H, K, V, monkeypatch):
    """Few heads and a long sequence: the state pass splits the chunks into
    segments (local passes + transitions, an fp32 scan, a final pass).  Slow
    decay carries the state across segment boundaries; the result must match
    the fp32 oracle and the one-segment pass."""
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    from oracle import gdn as og
    q, k, v, g, beta, h0 = _seg_inputs(T, H, K, V, seed=21)
    oref, sref = og.gdn_chunk(q, k, v, g, beta, None, h0, True, use_qk_l2norm=False)
    c = lambda x, dt=torch.bfloat16: x.to('cuda', dt)  # noqa: E731
    args = (c(q), c(k), c(v), c(g, torch.float32), c(beta))
    o, s = chunk_gated_delta_rule(*args, initial_state=c(h0, torch.float32), output_final_state=True)
    assert max_rel(o, oref) <= O_TOL and max_rel(s, sref) <= S_TOL
    monkeypatch.setenv('KB200_GDN_SEGMENTS', '1')
    o1, s1 = chunk_gated_delta_rule(*args, initial_state=c(h0, torch.float32), output_final_state=True)
    assert max_rel(o, o1) <= 1e-2 and max_rel(s, s1) <= 5e-3


def test_gdn_segmented_rank_share_of_config1():
    """One Ulysses rank's share of config 1 at 8 GPUs (T=32760, 3 heads), the
    case the segmented state pass exists for; two heads against the oracle."""
    from kairos_sensenova_b200 import chunk_gated_delta_rule
    from kairos_sensenova_b200.inputs import gdn_inputs
    from oracle import gdn as og
    q, k, v, g, beta = gdn_inputs(1, 32760, 3, 128, 128, seed=0, device='cuda')
    o, s = chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True, use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    for h in (0, 2):
        sl = lambda x: x[:, :, h:h + 1].float().cpu()  # noqa: E731
        oref, sref = og.gdn_chunk(sl(q), sl(k), sl(v), sl(g), sl(beta), None, None, True, use_qk_l2norm=True)
        assert max_rel(o[:, :, h:h + 1], oref) <= O_TOL
        assert max_rel(s[:, h:h + 1], sref) <= S_TOL
