"""Ulysses sequence<->head re-partition over NCCL (NVLink / NVSwitch).

Same names, arguments, return values and errors as the reference
(``kairos/modules/utils/tp_utils.py:84-254``):

* ``all2all_seq_to_head(x, context_group, tp_chunk_list=None, head_dim=None)``:
  ``[B, N/P, D]`` -> ``[B, N, D_local]``, rank r receiving its head block of
  every rank's tokens (balanced: ``D_local = D/P``; unbalanced: rank r owns
  ``tp_chunk_list[r]`` heads of ``head_dim`` channels);
* ``all2all_head_to_seq(x, context_group, tp_chunk_list=None, head_dim=None)``:
  the inverse, ``[B, N, D_local]`` -> ``[B, N/P, D]``;
* both return ``x`` unchanged when torch.distributed is not initialised or the
  group has one rank, and raise ``RuntimeError`` on indivisible shapes.

Instead of the reference's list-form ``dist.all_to_all`` plus ``torch.cat``
copies, each direction packs one contiguous ``[P, B, rows, cols]`` buffer,
issues a single ``dist.all_to_all_single`` (one NCCL grouped send/recv over
NVLink; also supported by gloo, which lacks the list form), and unpacks with
one strided copy.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _world_rank(group):
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    world = dist.get_world_size(group=group) if group is not None else dist.get_world_size()
    rank = dist.get_rank(group=group) if group is not None else dist.get_rank()
    return world, rank


def _chunks(tp_chunk_list, head_dim, world, d_full):
    if head_dim is None:
        raise RuntimeError("head_dim must be provided when tp_chunk_list is not None")
    if len(tp_chunk_list) != world:
        raise RuntimeError(f"len(tp_chunk_list)={len(tp_chunk_list)} != world={world}")
    if any(int(v) <= 0 for v in tp_chunk_list):
        raise RuntimeError(f"tp_chunk_list must be positive ints, got {tp_chunk_list}")
    dims = [int(v) * int(head_dim) for v in tp_chunk_list]
    if d_full is not None and sum(dims) != d_full:
        raise RuntimeError(f"sum(dim_chunk_list)={sum(dims)} != D_full={d_full}, "
                           f"tp_chunk_list={tp_chunk_list}, head_dim={head_dim}")
    return dims


def all2all_seq_to_head(x: torch.Tensor, context_group, tp_chunk_list=None, head_dim=None):
    world, rank = _world_rank(context_group)
    if world <= 1:
        return x
    B, N_local, D_full = x.shape
    if tp_chunk_list is None:
        if D_full % world != 0:
            raise RuntimeError(f"D_full={D_full} must be divisible by world={world}")
        D_local = D_full // world
        send = x.reshape(B, N_local, world, D_local).permute(2, 0, 1, 3).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=context_group)
        # recv[src] = src's tokens for my heads -> [B, world*N_local, D_local]
        return recv.permute(1, 0, 2, 3).reshape(B, world * N_local, D_local)
    dims = _chunks(tp_chunk_list, head_dim, world, D_full)
    dmax = max(dims)
    send = x.new_zeros(world, B, N_local, dmax)
    off = 0
    for r, d in enumerate(dims):
        send[r, :, :, :d] = x[:, :, off:off + d]
        off += d
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=context_group)
    return recv[..., :dims[rank]].permute(1, 0, 2, 3).reshape(B, world * N_local, dims[rank])


def all2all_head_to_seq(x: torch.Tensor, context_group, tp_chunk_list=None, head_dim=None):
    world, rank = _world_rank(context_group)
    if world <= 1:
        return x
    B, N_full, D_local = x.shape
    if N_full % world != 0:
        raise RuntimeError(
            f"all2all_head_to_seq currently only supports seq evenly divisible by world size, "
            f"got N_full={N_full}, world={world}")
    N_local = N_full // world
    if tp_chunk_list is None:
        send = x.reshape(B, world, N_local, D_local).permute(1, 0, 2, 3).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=context_group)
        # recv[src] = my tokens of src's heads -> [B, N_local, world*D_local]
        return recv.permute(1, 2, 0, 3).reshape(B, N_local, world * D_local)
    dims = _chunks(tp_chunk_list, head_dim, world, None)
    if D_local % head_dim != 0:
        raise RuntimeError(f"D_local={D_local} must be divisible by head_dim={head_dim}")
    if D_local != dims[rank]:
        raise RuntimeError(f"D_local={D_local}, expected {dims[rank]}")
    dmax = max(dims)
    send = x.new_zeros(world, B, N_local, dmax)
    send[..., :D_local] = x.reshape(B, world, N_local, D_local).permute(1, 0, 2, 3)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=context_group)
    return torch.cat([recv[r, :, :, :dims[r]] for r in range(world)], dim=2)
