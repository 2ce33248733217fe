"""Failure detection on the host (no GPU): a rank that leaves between steps.

Two gloo ranks run the Ulysses re-partition (all2all_seq_to_head /
all2all_head_to_seq) for a step; then rank 1 exits without joining the next
step.  Rank 0's next exchange must end with an error within the process
group's (short) timeout instead of hanging, and rank 0 reports it.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _send(q, item):
    q.put(item)
    q.close()
    q.join_thread()      # flushed before the process ends abruptly


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    from kairos_sensenova_b200.ulysses import all2all_head_to_seq, all2all_seq_to_head
    x = torch.randn(1, 8, 4 * 16) + rank
    y = all2all_seq_to_head(x, None, head_dim=16)
    z = all2all_head_to_seq(y, None, head_dim=16)
    ok_step = bool(torch.equal(z, x))
    dist.barrier()
    if rank == 1:
        _send(q, (rank, 'left', ok_step))
        os._exit(0)                     # leaves between steps, with no collective in flight
    t0 = time.time()
    try:
        all2all_seq_to_head(x, None, head_dim=16)
        _send(q, (rank, 'no error', ok_step))
    except Exception as e:  # the peer is gone: gloo reports it (closed connection or timeout)
        _send(q, (rank, f'error after {time.time() - t0:.1f}s: {type(e).__name__}', ok_step))
    os._exit(0)


@pytest.mark.timeout(120)
def test_rank_leaving_between_steps_is_reported_not_hung():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, msg, ok_step = q.get(timeout=90)
        res[rank] = (msg, ok_step)
    for p in procs:
        p.join(timeout=30)
    assert res[0][1] and res[1][1]                    # the step before the failure was right
    assert res[1][0] == 'left'
    assert res[0][0].startswith('error after'), res[0][0]
    secs = float(res[0][0].split()[2].rstrip('s:'))
    assert secs < 60                                  # ended well inside the test budget
