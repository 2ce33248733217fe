"""Ulysses all-to-all wrapper on CPU gloo ranks (world 2 and 3), checked
against the index arithmetic of the reference's semantics (oracle.layers),
and the mixers' slabbed projection exchange against a plain product."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
        dist.init_process_group('gloo', rank=rank, world_size=world)
        from kairos_sensenova_b200.ulysses import all2all_head_to_seq, all2all_seq_to_head
        from oracle.layers import head_to_seq_expected, seq_to_head_expected
        g = torch.Generator().manual_seed(0)
        B, N, hd = 2, 6 * world, 4
        H = 2 * world
        full = torch.randn(B, N, H * hd, generator=g)
        n = N // world
        x = full[:, rank * n:(rank + 1) * n].clone()
        y = all2all_seq_to_head(x, None)
        assert torch.equal(y, seq_to_head_expected(full, rank, world))
        z = all2all_head_to_seq(y, None)
        assert torch.equal(z, x)                                   # round trip is exact
        assert torch.equal(all2all_head_to_seq(full[..., rank * 2 * hd:(rank + 1) * 2 * hd].clone(), None),
                           head_to_seq_expected(full, rank, world)[..., :] if world == 1 else
                           torch.cat([full[:, rank * n:(rank + 1) * n, r * 2 * hd:(r + 1) * 2 * hd]
                                      for r in range(world)], dim=2))
        # unbalanced heads: rank r owns r+1 heads
        chunks = [r + 1 for r in range(world)]
        Hu = sum(chunks)
        fu = torch.randn(B, N, Hu * hd, generator=g)
        xu = fu[:, rank * n:(rank + 1) * n].clone()
        yu = all2all_seq_to_head(xu, None, tp_chunk_list=chunks, head_dim=hd)
        dims = [c * hd for c in chunks]
        assert torch.equal(yu, seq_to_head_expected(fu, rank, world, dims))
        assert torch.equal(all2all_head_to_seq(yu, None, tp_chunk_list=chunks, head_dim=hd), xu)
        # error behaviour matches the reference
        with pytest.raises(RuntimeError):
            all2all_seq_to_head(torch.zeros(1, 2, world * 3 + 1), None)
        with pytest.raises(RuntimeError):
            all2all_head_to_seq(torch.zeros(1, world + 1, 4), None)
        with pytest.raises(RuntimeError):
            all2all_seq_to_head(xu, None, tp_chunk_list=chunks, head_dim=None)
        # slabbed projection + seq->head exchange of the mixers (destination-grouped
        # GEMM per token slab, grouped sends/receives): rank r ends up with
        # x_full @ W[r] (+ b[r]) in global token order; `post` sees each slab
        from kairos_sensenova_b200.mixers import _Ulysses
        T, hid, C = 12 * world, 8, 5
        xf = torch.randn(T, hid, generator=g)
        W = torch.randn(world, hid, C, generator=g)
        b = torch.randn(world, C, generator=g)
        Tl = T // world
        u = _Ulysses(2 * world, 4, world, rank, None)
        u.slabs = 3
        seen = []

        def post(send, r0):
            seen.append((r0, send.shape[1]))
            send[..., 0] = send[..., 0] + (rank * Tl + r0 + torch.arange(send.shape[1])).float()

        got = u._project_exchange(xf[rank * Tl:(rank + 1) * Tl].clone(), W, b, post)
        want = xf @ W[rank] + b[rank]
        want[:, 0] += torch.arange(T).float()
        assert got.shape == (T, C) and torch.allclose(got, want, atol=1e-5), (got - want).abs().max()
        assert seen == [(0, 4), (4, 4), (8, 4)]
        dist.barrier()
        q.put((rank, 'ok'))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize('world', [2, 3])
def test_ulysses_gloo(world):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == 'ok' for v in res.values()), res


def test_ulysses_single_process_is_identity():
    from kairos_sensenova_b200.ulysses import all2all_head_to_seq, all2all_seq_to_head
    x = torch.randn(1, 4, 8)
    assert all2all_seq_to_head(x, None) is x
    assert all2all_head_to_seq(x, None) is x
