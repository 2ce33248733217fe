"""The benchmark's hybrid block (P = 1) against the CPU oracle chain."""
import pytest
import torch

from conftest import max_rel

pytestmark = pytest.mark.gpu


def test_hybrid_block_matches_oracle():
    from kairos_sensenova_b200.hybrid import HybridBlock
    from oracle.hybrid import attn_chain, freqs_cis_3d, gdn_chain, weights_of
    H, D, hidden, T = 4, 128, 512, 300
    blk = HybridBlock(hidden=hidden, heads=H, head_dim=D, seed=5, grid=(3, 10, 10))
    blk.nq.uniform_(0.5, 1.5)
    blk.nk.uniform_(0.5, 1.5)
    w = weights_of(blk)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(T, hidden, generator=gen).bfloat16()
    y = blk.gdn_chain(x.cuda())
    yr = gdn_chain(w, x.float(), H, D)
    assert max_rel(y, yr) < 3e-2
    z = blk.attn_chain(y)
    zr = attn_chain(w, y.float().cpu(), H, D, freqs=freqs_cis_3d(D, 3, 10, 10))
    c = torch.nn.functional.cosine_similarity(z.float().cpu().flatten(), zr.flatten(), dim=0).item()
    assert c >= 0.999
