"""Host-side logic that needs no GPU: the device-built varlen chunk table (run
here on CPU tensors), the layer cache object and the conv-state carry."""
import torch

from kairos_sensenova_b200.gated_delta_rule import prepare_chunk_indices
from kairos_sensenova_b200.layers import Cache, _next_conv_state


def _host_table(lens, bt=64):
    pairs, offs = [], [0]
    for n, ln in enumerate(lens):
        nt = (ln + bt - 1) // bt
        pairs += [(n, i) for i in range(nt)]
        offs.append(offs[-1] + nt)
    return pairs, offs


def test_chunk_table_matches_host_enumeration():
    for lens in ([1, 63, 64, 65, 200], [0, 5, 0], [4096], [1] * 9, [130, 0, 64]):
        cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()))
        idx, offs, M = prepare_chunk_indices(cu, int(cu[-1]))
        pairs, hoffs = _host_table(lens)
        assert M == (sum(lens) + 63) // 64 + len(lens) >= len(pairs)
        assert offs.tolist() == hoffs
        assert idx[:len(pairs)].tolist() == [list(p) for p in pairs]
        assert (idx[len(pairs):, 0] == -1).all()
        assert idx.dtype == torch.int32 and offs.dtype == torch.int32


def test_cache_follows_fla_cache_semantics():
    c = Cache.from_legacy_cache()
    assert len(c) == 0 and c.get_seq_length() == 0
    st = c.update(recurrent_state=torch.ones(1), conv_state=(1, 2, 3), layer_idx=2, offset=10)
    assert len(c) == 3 and c[2] is st and c[0]['recurrent_state'] is None
    assert c.get_seq_length(0) == 0                 # only layer 0 counts tokens (FLACache)
    c.update(recurrent_state=torch.zeros(1), layer_idx=0, offset=7)
    assert c.get_seq_length(0) == 7
    c.update(conv_state=None, layer_idx=2, offset=5)  # None leaves the stored state alone
    assert c[2]['conv_state'] == (1, 2, 3)
    c2 = Cache.from_legacy_cache(c.to_legacy_cache())
    assert len(c2) == 3 and c2[2]['conv_state'] == (1, 2, 3)


def test_next_conv_state_is_the_last_w_inputs():
    W, C = 4, 6
    seq = torch.randn(1, 11, C)
    state = None
    for s, e in ((0, 1), (1, 3), (3, 8), (8, 11)):
        state = _next_conv_state(state, seq[:, s:e], W)
        want = torch.zeros(1, C, W)
        n = min(W, e)
        want[..., W - n:] = seq[0, e - n:e].t()
        assert torch.equal(state, want), (s, e)
