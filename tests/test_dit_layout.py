"""Host-side layout of the DiT step (no GPU): the patch embedding as a GEMM
over flattened patches equals the reference's Conv3d, and unpatchify is the
reference's rearrange (``kairos_dit.py:1167-1181``); the mixer patterns."""
from types import SimpleNamespace

import torch
import torch.nn.functional as F
from einops import rearrange

from kairos_sensenova_b200.dit import DiTConfig, KairosDiT, sinusoidal_embedding_1d


def _fake(cfg, world=1, rank=0):
    return SimpleNamespace(cfg=cfg, P=world, rank=rank)


def test_patchify_is_the_conv3d_patch_embedding():
    cfg = DiTConfig(dim=32, heads=1, latent=(3, 8, 6))
    gen = torch.Generator().manual_seed(0)
    lat = torch.randn(cfg.in_dim, *cfg.latent, generator=gen)
    W = torch.randn(cfg.dim, cfg.in_dim, *cfg.patch, generator=gen)
    b = torch.randn(cfg.dim, generator=gen)
    p = KairosDiT._patchify(_fake(cfg), lat.bfloat16().float()).float()
    got = p @ W.reshape(cfg.dim, -1).t() + b
    ref2 = F.conv3d(lat.bfloat16().float()[None], W, b, stride=cfg.patch)[0].flatten(1).t()
    assert got.shape == ref2.shape == (cfg.tokens, cfg.dim)
    assert torch.allclose(got, ref2, atol=1e-4, rtol=1e-4)
    # each rank gets its contiguous token shard
    shards = [KairosDiT._patchify(_fake(cfg, 2, r), lat) for r in range(2)]
    assert torch.equal(torch.cat(shards), KairosDiT._patchify(_fake(cfg), lat))


def test_unpatchify_is_the_reference_rearrange():
    cfg = DiTConfig(dim=32, heads=1, latent=(3, 8, 6))
    f, h, w = cfg.grid
    y = torch.randn(f * h * w, cfg.out_dim * 4)
    ref = rearrange(y[None], 'b (f h w) (x y z c) -> b c (f x) (h y) (w z)', f=f, h=h, w=w, x=1, y=2, z=2)[0]
    assert torch.equal(KairosDiT._unpatchify(_fake(cfg), y), ref)


def test_mixer_patterns_and_sinusoid():
    base, ref = DiTConfig(layers=8), DiTConfig(layers=8, pattern='reference')
    assert [base.is_gdn(i) for i in range(8)] == [True, True, True, False] * 2
    assert [ref.is_gdn(i) for i in range(8)] == [False, False, False, True] * 2
    e = sinusoidal_embedding_1d(256, torch.tensor([0.0, 500.0]))
    assert e.shape == (2, 256) and torch.equal(e[0, :128], torch.ones(128, dtype=torch.float64))
    assert abs(float(e[1, 0]) - float(torch.cos(torch.tensor(500.0, dtype=torch.float64)))) < 1e-12


def test_oracle_block_matches_reference_dit_block():
    """The DiT oracle's block against the reference's own ``DiTBlock`` run on
    CPU (fixture from ``tests/golden/make_dit_golden.py``): modulation order,
    gated residuals, cross-attention norms and FFN are the reference's.  The
    oracle rounds the normalised, rotated q/k to bf16 as the GPU path does
    (the reference's fp32 run does not); agreement is ~3e-5, while swapping
    scale and shift or the FFN activation moves the output by 2e-3 - 3e-3."""
    from conftest import GOLDEN
    from oracle.dit import block_weights_from_reference, dit_block
    d = torch.load(GOLDEN / 'dit_block_attn.pt')
    b = block_weights_from_reference(d['state_dict'])
    H, D = d['heads'], d['dim']
    y = dit_block(b, d['x'][0], d['context'][0], d['t_mod'][0], H, D // H, d['eps'], d['grid'], False, 'silu')
    ref = d['out'][0]
    err = float((y - ref).abs().max() / ref.abs().max())
    assert err < 5e-4, err


def test_oracle_gdn_block_matches_reference_dit_block():
    """The GatedDeltaNet branch of the reference's own ``DiTBlock`` run on CPU
    (fixture from ``tests/golden/make_dit_gdn_golden.py``: the block's single-device
    walk in T/8 pieces through one FLA Cache, ``kairos_dit.py:857-922``): (a) the
    one-shot layer oracle on the branch's whole input equals the reference's
    chunked walk; (b) the DiT oracle's GDN block (modulation, gated residual,
    cross-attention, FFN around ``oracle.hybrid.gdn_chain``) equals the block output."""
    from conftest import GOLDEN
    from oracle import layers as ol
    from oracle.dit import block_weights_from_reference, dit_block
    d = torch.load(GOLDEN / 'dit_block_gdn.pt')
    sd = d['state_dict']
    gsd = {k[len('gated_delta.'):]: v for k, v in sd.items() if k.startswith('gated_delta.')}
    H, hd, eps = d['heads'], d['head_dim'], d['eps']
    one_shot = ol.gated_deltanet_forward(gsd, d['gdn_in'], H, hd, hd, eps, emulate_bf16=False)
    err = float((one_shot - d['gdn_out']).abs().max() / d['gdn_out'].abs().max())
    assert err < 1e-4, err
    b = block_weights_from_reference(sd)
    b.update({'Wq': gsd['q_proj.weight'], 'Wk': gsd['k_proj.weight'], 'Wv': gsd['v_proj.weight'],
              'Wa': gsd['a_proj.weight'], 'Wb': gsd['b_proj.weight'], 'Wg': gsd['g_proj.weight'],
              'Wo': gsd['o_proj.weight'], 'cq': gsd['q_conv1d.weight'][:, 0], 'ck': gsd['k_conv1d.weight'][:, 0],
              'cv': gsd['v_conv1d.weight'][:, 0], 'A_log': gsd['A_log'], 'dt_bias': gsd['dt_bias'],
              'o_norm_w': gsd['o_norm.weight']})
    y = dit_block(b, d['x'][0], d['context'][0], d['t_mod'][0], H, hd, eps, d['grid'], True, 'silu')
    ref = d['out'][0]
    err = float((y - ref).abs().max() / ref.abs().max())
    assert err < 5e-4, err
