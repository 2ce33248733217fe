"""Sequence-parallel paths on 2 GPUs (NCCL, one process per GPU): the hybrid
block and a small DiT step sharded over two ranks must match the same model
run on one GPU, and the hybrid block and the DiT step captured as CUDA graphs
(NCCL sends and receives inside) must match their eager runs; the graphs are
destroyed before the process group on every rank.  Skipped on boxes with fewer than
two GPUs.

Tolerances: the sharded run changes only the GEMM shapes, the per-rank head
split of the GDN state pass (V-slice width, segment count) and the order of
NCCL transfers, so the outputs agree to bf16 level: max-relative error
<= 2e-2 and cosine similarity >= 0.9995.
"""
import datetime
import gc
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cmp(a, b):
    a, b = a.float().flatten().cpu(), b.float().flatten().cpu()
    cos = float(torch.dot(a, b) / (a.norm() * b.norm()))
    return float((a - b).abs().max() / b.abs().max()), cos


def _worker(rank, world, port, q):
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group('nccl', rank=rank, world_size=world, device_id=torch.device('cuda', rank),
                                timeout=datetime.timedelta(seconds=120))
        from kairos_sensenova_b200.dit import DiTConfig, KairosDiT, make_weights
        from kairos_sensenova_b200.hybrid import HybridBlock
        res = {}
        with torch.no_grad():
            T, hid, H = 4096, 768, 6
            gen = torch.Generator(device='cuda').manual_seed(4)
            xf = torch.randn(T, hid, generator=gen, device='cuda').bfloat16()
            Tl = T // world
            ref = HybridBlock(hid, H, 128, grid=(4, 32, 32)).forward(xf)
            blk = HybridBlock(hid, H, 128, world=world, rank=rank, grid=(4, 32, 32))
            y = blk.forward(xf[rank * Tl:(rank + 1) * Tl].contiguous())
            res['hybrid'] = _cmp(y, ref[rank * Tl:(rank + 1) * Tl])
            from kairos_sensenova_b200.graphs import GraphedStep
            xg = xf[rank * Tl:(rank + 1) * Tl].contiguous()
            gstep = GraphedStep(blk.forward, xg)       # NCCL sends/receives captured in the graph
            yg = gstep(xg).clone()
            torch.cuda.synchronize()
            res['hybrid_graph'] = _cmp(yg, y)
            del gstep                                  # graphs go before the process group does
            cfg = DiTConfig(dim=256, heads=2, ffn_dim=512, layers=4, text_dim=64, text_len=16, latent=(4, 16, 16))
            w = make_weights(cfg, 'cuda', seed=2)
            g2 = torch.Generator(device='cuda').manual_seed(7)
            lat = torch.randn(cfg.in_dim, *cfg.latent, generator=g2, device='cuda')
            ctx = torch.randn(cfg.text_len, cfg.text_dim, generator=g2, device='cuda')
            t = torch.tensor([500.0], device='cuda')
            o1 = KairosDiT(cfg, weights=w)(lat, t, ctx)
            o2 = KairosDiT(cfg, world=world, rank=rank, weights=w)(lat, t, ctx)
            res['dit'] = _cmp(o2, o1)
            m2 = KairosDiT(cfg, world=world, rank=rank, weights=w)
            dstep = GraphedStep(m2, lat, t, ctx)
            o3 = dstep(lat, t, ctx).clone()
            torch.cuda.synchronize()
            res['dit_graph'] = _cmp(o3, o2)
            del dstep
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, res))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason='needs 2 GPUs')
def test_sequence_parallel_two_gpus_match_one():
    world = 2
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, r in res.items():
        assert isinstance(r, dict), r
        for name, (mr, cos) in r.items():
            assert mr <= 2e-2 and cos >= 0.9995, (rank, name, mr, cos)
