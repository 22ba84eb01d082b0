"""Multi-GPU partition of the attention backward over (batch, kv-head) units.

The reference evaluates on one GPU (eval_modal_attn_bwd.py:70) and has no
parallel scheme.  Here the bs·8 units u = b*8 + kv_head are independent: unit u
reads dO[b,:,10kvh:10kvh+10], the 10 heads of P / P_drop / mask and V[b,kvh],
and writes those 10 heads of dS and dV[b,kvh].  Each rank computes a
contiguous range of units with no exchange; the only collective is the
optional gather of the shards to rank 0 at the end (point-to-point send/recv,
NCCL over NVLink on GPUs, gloo on CPU for the host-side tests).
"""
import torch
import torch.distributed as dist

KVH, G, H, D = 8, 10, 80, 128


def unit_range(n_units, rank, world):
    """Contiguous, balanced split of [0, n_units) (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    return n_units * rank // world, n_units * (rank + 1) // world


def head_slice(u0, u1):
    """Flattened (batch*80 + head) range of the heads of units [u0, u1)."""
    return u0 * G, u1 * G


def shard_inputs(data, u0, u1):
    """Cuts the shard of the reference tuple: full dO and V, the units' heads of
    P / P_drop / mask as [(u1-u0)*10, sq, skv] views (no copy when contiguous)."""
    dO, P, Pd, V, M, p = data
    bs, _, sq, skv = P.shape
    h0, h1 = head_slice(u0, u1)
    flat = lambda t: t.reshape(bs * H, sq, skv)[h0:h1]
    return dO, flat(P), flat(Pd), V, flat(M), p


def gather_to_rank0(dS_shard, dV_shard, bs, sq, skv, group=None):
    """Collects every rank's (dS_shard, dV_shard) into full [bs,80,sq,skv] and
    [bs,8,skv,128] tensors on rank 0 (returns None elsewhere).  Shards must be
    the unit_range() split of bs*8 units over the group."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n_units = bs * KVH
    if rank != 0:
        dist.send(dS_shard.contiguous(), dst=0, group=group)
        dist.send(dV_shard.contiguous(), dst=0, group=group)
        return None
    dS = torch.empty(bs * H, sq, skv, dtype=dS_shard.dtype, device=dS_shard.device)
    dV = torch.empty(bs * KVH, skv, D, dtype=dV_shard.dtype, device=dV_shard.device)
    for r in range(world):
        u0, u1 = unit_range(n_units, r, world)
        h0, h1 = head_slice(u0, u1)
        if r == 0:
            dS[h0:h1].copy_(dS_shard)
            dV[u0:u1].copy_(dV_shard)
        else:
            dist.recv(dS[h0:h1], src=r, group=group)
            dist.recv(dV[u0:u1], src=r, group=group)
    return dS.view(bs, H, sq, skv), dV.view(bs, KVH, skv, D)
