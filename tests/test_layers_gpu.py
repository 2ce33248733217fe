"""GPU parity of the prologue / epilogue fusion kernels and the GatedDeltaNet
layer drop-in against the CPU oracle (oracle.layers)."""
import pytest
import torch

from conftest import max_rel
from oracle import layers as ol

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('T', [1, 3, 70, 513])
def test_prologue_matches_oracle(T):
    from kairos_sensenova_b200.fused_ops import gdn_prologue
    gen = torch.Generator().manual_seed(T)
    B, H, K, V = 2, 3, 128, 256
    xq = torch.randn(B * T, H * K, generator=gen).bfloat16()
    xk = torch.randn(B * T, H * K, generator=gen).bfloat16()
    xv = torch.randn(B * T, H * V, generator=gen).bfloat16()
    a = torch.randn(B * T, H, generator=gen).bfloat16()
    b = torch.randn(B * T, H, generator=gen).bfloat16()
    wq, wk, wv = (torch.randn(c, 4, generator=gen) * 0.5 for c in (H * K, H * K, H * V))
    A_log = torch.rand(H, generator=gen) * 2
    dt_bias = torch.randn(H, generator=gen)
    c = lambda t: t.cuda()  # noqa: E731
    q, k, v, g, beta = gdn_prologue(c(xq), c(xk), c(xv), c(a), c(b), c(wq), c(wk), c(wv), c(A_log),
                                    c(dt_bias), H, B, T)
    ref = lambda x, w: ol.short_conv_silu(x.reshape(B, T, -1), w)  # noqa: E731
    assert max_rel(q.reshape(B, T, -1), ref(xq, wq)) < 1e-2
    assert max_rel(k.reshape(B, T, -1), ref(xk, wk)) < 1e-2
    assert max_rel(v.reshape(B, T, -1), ref(xv, wv)) < 1e-2
    gr, br = ol.gates(a, b, A_log, dt_bias)
    assert max_rel(g.reshape(-1, H), gr) < 1e-5
    assert max_rel(beta.reshape(-1, H), br) < 1e-2


def test_prologue_strided_fused_projection():
    """q/k/v/a/b given as column slices of one fused projection output."""
    from kairos_sensenova_b200.fused_ops import gdn_prologue
    gen = torch.Generator().manual_seed(1)
    B, T, H, K = 1, 100, 2, 128
    C = 3 * H * K + 2 * H + 4          # padded like the Ulysses-packed layout
    proj = torch.randn(T, C, generator=gen).bfloat16().cuda()
    w = torch.randn(H * K, 4, generator=gen).cuda()
    A_log, dtb = torch.zeros(H).cuda(), torch.zeros(H).cuda()
    s = lambda i: proj[:, i * H * K:(i + 1) * H * K]  # noqa: E731
    ab = 3 * H * K
    q, k, v, g, beta = gdn_prologue(s(0), s(1), s(2), proj[:, ab:ab + H], proj[:, ab + H:ab + 2 * H],
                                    w, w, w, A_log, dtb, H, B, T)
    q2, k2, v2, g2, b2 = gdn_prologue(s(0).contiguous(), s(1).contiguous(), s(2).contiguous(),
                                      proj[:, ab:ab + H].contiguous(), proj[:, ab + H:ab + 2 * H].contiguous(),
                                      w, w, w, A_log, dtb, H, B, T)
    for x, y in ((q, q2), (k, k2), (v, v2), (g, g2), (beta, b2)):
        assert torch.equal(x, y)


@pytest.mark.parametrize('D', [128, 256])
def test_rmsnorm_gated_matches_oracle(D):
    from kairos_sensenova_b200.fused_ops import rms_norm_gated
    gen = torch.Generator().manual_seed(D)
    x = torch.randn(5, 7, 3, D, generator=gen).bfloat16()
    gt = torch.randn(5, 7, 3, D, generator=gen).bfloat16()
    w = torch.rand(D, generator=gen) + 0.5
    y = rms_norm_gated(x.cuda(), gt.cuda(), w.cuda(), 1e-5)
    assert y.dtype == torch.bfloat16
    assert max_rel(y, ol.rmsnorm_gated(x, gt, w, 1e-5)) < 1e-2


def test_gated_deltanet_layer_matches_oracle():
    from kairos_sensenova_b200.layers import GatedDeltaNet
    torch.manual_seed(0)
    hidden, H, hd = 512, 4, 128
    layer = GatedDeltaNet(hidden_size=hidden, expand_v=1, head_dim=hd, num_heads=H)
    with torch.no_grad():
        for n, p_ in layer.named_parameters():
            if n.endswith('proj.weight'):
                p_.normal_(0, 0.02)
    sd = {k: v.detach().clone() for k, v in layer.state_dict().items()}
    layer = layer.cuda().to(torch.bfloat16)
    x = torch.randn(1, 300, hidden).bfloat16()
    with torch.no_grad():
        o, _, _ = layer(x.cuda())
    ref = ol.gated_deltanet_forward({k: v.bfloat16().float() for k, v in sd.items()}, x.float(), H, hd, hd)
    assert o.shape == (1, 300, hidden)
    assert max_rel(o, ref) < 2e-2


@pytest.mark.parametrize('H', [3, 4, 24])   # 384 channels: CTA-per-rows form; 512, 3072: warp-per-row form
def test_rmsnorm_rope_matches_reference_math(H):
    from kairos_sensenova_b200.fused_ops import freqs_cis_3d, rmsnorm_rope, rope_table
    gen = torch.Generator().manual_seed(40)
    D = 128
    fr = freqs_cis_3d(D, 3, 5, 7)                      # 105 tokens on a 3x5x7 grid
    S = fr.shape[0]
    x = (torch.randn(1, S, H * D, generator=gen) * 3).bfloat16()
    w = torch.rand(H * D, generator=gen) + 0.5
    y = rmsnorm_rope(x.cuda(), w.cuda(), rope_table(fr, 'cuda'), D)
    ref = ol.rmsnorm_rope(x, w, fr, H)
    assert max_rel(y, ref) < 1e-2


@pytest.mark.parametrize('P,Hl', [(2, 2), (8, 3)])
def test_rmsnorm_rope_in_place_on_grouped_projection(P, Hl):
    """q as the first column block of a destination-grouped [P, T, 3*Hl*D] buffer."""
    from kairos_sensenova_b200.fused_ops import freqs_cis_3d, rmsnorm_rope, rope_table
    gen = torch.Generator().manual_seed(41)
    D, T = 128, 60
    buf = torch.randn(P, T, 3 * Hl * D, generator=gen).bfloat16().cuda()
    fr = freqs_cis_3d(D, 3, 4, 5)
    cs = rope_table(fr, 'cuda')
    q_full = torch.cat([buf[r, :, :Hl * D] for r in range(P)], dim=1)   # [T, P*Hl*D]
    ref = rmsnorm_rope(q_full.unsqueeze(0).contiguous(), None, cs, D)[0]
    rmsnorm_rope(buf, None, cs, D, out=buf, rows=T, dim=P * Hl * D, ld=3 * Hl * D, heads_per_block=Hl,
                 block_stride=T * 3 * Hl * D)
    got = torch.cat([buf[r, :, :Hl * D] for r in range(P)], dim=1)
    assert torch.equal(got, ref)


@pytest.mark.parametrize('pieces', [8, 'ragged'])
def test_gated_deltanet_cache_walk_matches_one_shot(pieces):
    """The DiT block's GDN loop (``kairos_dit.py:880-922``): the sequence walked in
    pieces through one Cache with use_cache=True gives the one-shot output (conv
    states carry the last W-1 projection inputs, the recurrent state carries
    through ``initial_state``/``output_final_state``); the final recurrent state
    equals the one-shot final state.  Tolerance 2e-2 max-relative."""
    from kairos_sensenova_b200.layers import Cache, GatedDeltaNet
    torch.manual_seed(1)
    hidden, H, hd, T = 512, 4, 128, 640
    layer = GatedDeltaNet(hidden_size=hidden, expand_v=1, head_dim=hd, num_heads=H, layer_idx=2)
    with torch.no_grad():
        for n, p_ in layer.named_parameters():
            if n.endswith('proj.weight'):
                p_.normal_(0, 0.02)
    layer = layer.cuda().to(torch.bfloat16)
    x = torch.randn(1, T, hidden, device='cuda').bfloat16()
    with torch.no_grad():
        full, _, c1 = layer(x, past_key_values=Cache(), use_cache=True)
        bounds = list(range(0, T + 1, T // 8)) if pieces == 8 else [0, 1, 3, 67, 130, 131, 400, T]
        cache = Cache.from_legacy_cache()
        outs = []
        for s, e in zip(bounds[:-1], bounds[1:]):
            o, _, cache = layer(x[:, s:e].contiguous(), past_key_values=cache, use_cache=True)
            outs.append(o)
    walk = torch.cat(outs, 1)
    assert max_rel(walk, full) < 2e-2
    assert cache.get_seq_length(0) == 0 and len(cache) == 3          # layer 2's state only, as FLACache
    assert max_rel(cache[2]['recurrent_state'], c1[2]['recurrent_state']) < 1e-2
    for a, b in zip(cache[2]['conv_state'], c1[2]['conv_state']):
        assert torch.equal(a, b)
    # without a cache the layer is the one-shot call
    with torch.no_grad():
        o0, _, none = layer(x)
    assert none is None and torch.equal(o0, full)


def test_reference_dit_block_gdn_walk_through_drop_in():
    """The reference ``DiTBlock``'s own GDN walk (fixture from
    ``tests/golden/make_dit_gdn_golden.py``: the modulated input in 8 pieces through
    one FLA Cache, ``kairos_dit.py:857-922``) replayed through the drop-in
    ``layers.GatedDeltaNet`` + ``layers.Cache`` on the GPU in bf16: the gathered
    output matches the reference's within 2e-2 max-relative."""
    from conftest import GOLDEN
    from kairos_sensenova_b200.layers import Cache, GatedDeltaNet
    d = torch.load(GOLDEN / 'dit_block_gdn.pt')
    gsd = {k[len('gated_delta.'):]: v for k, v in d['state_dict'].items() if k.startswith('gated_delta.')}
    layer = GatedDeltaNet(hidden_size=d['dim'], expand_v=1, head_dim=d['head_dim'], num_heads=d['heads'],
                          mode='chunk', use_gate=True, norm_eps=d['eps'], layer_idx=0)
    layer.load_state_dict(gsd)
    layer = layer.cuda().to(torch.bfloat16)
    x = d['gdn_in'].cuda().bfloat16()
    T, n = x.shape[1], d['pieces']
    cache = Cache.from_legacy_cache()
    outs = []
    with torch.no_grad():
        for s in range(0, T, T // n):
            o, _, cache = layer(x[:, s:s + T // n].contiguous(), past_key_values=cache, use_cache=True)
            outs.append(o)
    got = torch.cat(outs, 1).float().cpu()
    assert max_rel(got, d['gdn_out']) < 2e-2
