"""The CPU oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference's naive recurrence and its
Triton chunk kernels run under the Triton interpreter)."""
import glob

import pytest
import torch

from conftest import max_rel
from oracle import gdn as og

CASES = sorted(glob.glob(str(__import__('conftest').GOLDEN / 'gdn_*.pt')))


def _load(path):
    d = torch.load(path)
    f = lambda x: None if x is None else x.float()  # noqa: E731
    return d, f(d['q']), f(d['k']), f(d['v']), d['g'], f(d['beta']), d['h0']


def test_fixtures_present():
    names = {p.rsplit('/', 1)[-1] for p in CASES}
    for n in ('gdn_cfg0.pt', 'gdn_t1.pt', 'gdn_t63.pt', 'gdn_t64.pt', 'gdn_t65.pt', 'gdn_t1000.pt',
              'gdn_slowdecay.pt', 'gdn_b2.pt', 'gdn_k128v256.pt', 'gdn_k256v512.pt'):
        assert n in names


@pytest.mark.parametrize('path', CASES, ids=lambda p: p.rsplit('/', 1)[-1])
def test_reference_paths_agree(path):
    d = torch.load(path)
    assert d['meta']['agree_o'] < 1e-4 and d['meta']['agree_s'] < 1e-4
    assert max_rel(d['o_naive'], d['o_triton']) < 1e-2  # o_naive may be bf16-stored


@pytest.mark.parametrize('path', CASES, ids=lambda p: p.rsplit('/', 1)[-1])
def test_oracle_chunk_fp32_matches_reference(path):
    d, q, k, v, g, beta, h0 = _load(path)
    if d['meta']['T'] > 600:
        pytest.skip('large case covered by test_oracle_cfg0')
    o, s = og.gdn_chunk(q, k, v, g, beta, None, h0, True, use_qk_l2norm=True)
    assert max_rel(o, d['o_triton']) < 2e-5
    assert max_rel(s, d['s_triton']) < 2e-5


def test_oracle_cfg0():
    d, q, k, v, g, beta, h0 = _load(str(__import__('conftest').GOLDEN / 'gdn_cfg0.pt'))
    o, s = og.gdn_chunk(q, k, v, g, beta, None, h0, True, use_qk_l2norm=True)
    assert max_rel(o, d['o_triton']) < 2e-5
    assert max_rel(s, d['s_triton']) < 2e-5
    ob, sb = og.gdn_chunk(q, k, v, g, beta, None, h0, True, use_qk_l2norm=True, emulate_bf16=True)
    # the bf16 pipeline model sits well inside the GPU tolerance
    assert max_rel(ob, d['o_triton']) < 1e-2
    assert max_rel(sb, d["s_triton"]) < 1e-2


def test_oracle_recurrent_matches_chunk_fp64():
    g_ = torch.Generator().manual_seed(3)
    B, T, H, K, V = 2, 150, 2, 32, 48
    q, k = torch.randn(B, T, H, K, generator=g_, dtype=torch.float64), torch.randn(B, T, H, K, generator=g_, dtype=torch.float64)
    v = torch.randn(B, T, H, V, generator=g_, dtype=torch.float64)
    beta = torch.rand(B, T, H, generator=g_, dtype=torch.float64)
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, generator=g_, dtype=torch.float64))
    h0 = torch.randn(B, H, K, V, generator=g_, dtype=torch.float64)
    o1, s1 = og.gdn_recurrent(q, k, v, g, beta, 0.3, h0, True, True)
    o2, s2 = og.gdn_chunk(q, k, v, g, beta, 0.3, h0, True, True)
    assert (o1 - o2).abs().max() < 1e-12 and (s1 - s2).abs().max() < 1e-12


def test_oracle_varlen_equals_batched():
    g_ = torch.Generator().manual_seed(4)
    T1, T2, H, K, V = 70, 130, 2, 16, 16
    q, k = torch.randn(1, T1 + T2, H, K, generator=g_), torch.randn(1, T1 + T2, H, K, generator=g_)
    v = torch.randn(1, T1 + T2, H, V, generator=g_)
    beta, g = torch.rand(1, T1 + T2, H, generator=g_), -torch.rand(1, T1 + T2, H, generator=g_)
    cu = torch.tensor([0, T1, T1 + T2])
    o, s = og.gdn_chunk_varlen(q, k, v, g, beta, cu, None, None, True, True)
    oa, sa = og.gdn_chunk(q[:, :T1], k[:, :T1], v[:, :T1], g[:, :T1], beta[:, :T1], None, None, True, True)
    assert torch.allclose(o[:, :T1], oa, atol=1e-6) and torch.allclose(s[:1], sa, atol=1e-6)


def test_layer_oracle_matches_reference_gated_deltanet_layer():
    """The GatedDeltaNet layer oracle (short convolutions + SiLU, gates, chunk
    op, gated RMSNorm, projections) against the reference's own vendored layer
    run on CPU (fixture from ``tests/golden/make_layer_golden.py``)."""
    import torch
    from oracle import layers as ol
    d = torch.load(__import__('conftest').GOLDEN / 'layer_gdn.pt')
    y = ol.gated_deltanet_forward(d['state_dict'], d['x'], d['heads'], d['head_dim'], d['head_dim'],
                                  d['norm_eps'], emulate_bf16=False)
    ref = d['out']
    err = float((y - ref).abs().max() / ref.abs().max())
    assert err < 1e-4, err


def test_dit_rows_oracle_equals_full_oracle_on_its_rows():
    """oracle.dit.dit_forward_rows (used by the full-size config-4 block tests) is
    exact for the rows it computes: checked against the full-sequence oracle on a
    small one-block model of each mixer kind."""
    from kairos_sensenova_b200.dit import DiTConfig, make_weights
    from oracle.dit import dit_forward, dit_forward_rows, patch_rows
    for pat in ('baseline', 'reference'):
        cfg = DiTConfig(dim=256, heads=2, ffn_dim=512, layers=1, text_dim=64, text_len=16, latent=(4, 16, 16),
                        pattern=pat)
        w = make_weights(cfg, 'cpu', seed=2)
        gen = torch.Generator().manual_seed(7)
        lat = torch.randn(cfg.in_dim, *cfg.latent, generator=gen)
        ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=gen)
        t = torch.tensor([500.0])
        full = patch_rows(dit_forward(w, cfg, lat, t, ctx), cfg)
        rows = dit_forward_rows(w, cfg, lat, t, ctx, 100)
        assert (full[:100] - rows).abs().max() <= 1e-5 * full.abs().max()
