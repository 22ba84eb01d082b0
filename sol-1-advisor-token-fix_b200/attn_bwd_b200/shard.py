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


def unit_step(sq, skv):
    """Smallest g in {1, 2, 4, 8} for which g units (10·g heads of sq·skv elements) are a
    multiple of 16 elements: shard boundaries on multiples of g keep every slice of P /
    P_drop / mask / dS 16-byte aligned and keep the rows' alignment classes (the same rule
    as the C library's host-buffer pipeline)."""
    for g in (1, 2, 4):
        if (G * g * sq * skv) % 16 == 0:
            return g
    return 8


def unit_range(n_units, rank, world, sq=None, skv=None):
    """Contiguous, balanced split of [0, n_units).  Without (sq, skv) sizes differ by at
    most 1; with them, boundaries fall on multiples of unit_step(sq, skv), so that every
    rank's slices start 16-byte aligned and need no copy (sizes then differ by at most one
    step)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    g = 1 if sq is None or skv is None else unit_step(sq, skv)
    steps = (n_units + g - 1) // g
    return min(steps * rank // world * g, n_units), min(steps * (rank + 1) // world * g, n_units)


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


def gather_to_rank0(dS_shard, dV_shard, bs, sq, skv, group=None, out=None, aligned=True):
    """Collects every rank's (dS_shard, dV_shard) into full [bs,80,sq,skv] and
    [bs,8,skv,128] tensors on rank 0 (returns None elsewhere).  Shards must be the
    unit_range() split of bs*8 units over the group (aligned=True: the split with
    (sq, skv), as the multi-GPU path uses; False: the plain split).  ``out`` optionally
    supplies rank 0's (dS, dV) destination tensors.

    All transfers are posted as one batch of point-to-point operations, so every peer
    streams into rank 0 at the same time (NCCL runs them concurrently over NVLink)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n_units = bs * KVH
    rng = (lambda r: unit_range(n_units, r, world, sq, skv)) if aligned else (lambda r: unit_range(n_units, r, world))
    if rank != 0:
        ops = [dist.P2POp(dist.isend, dS_shard.contiguous(), 0, group),
               dist.P2POp(dist.isend, dV_shard.contiguous(), 0, group)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()
        return None
    if out is None:
        dS = torch.empty(bs * H, sq, skv, dtype=dS_shard.dtype, device=dS_shard.device)
        dV = torch.empty(bs * KVH, skv, D, dtype=dV_shard.dtype, device=dV_shard.device)
    else:
        dS = out[0].view(bs * H, sq, skv)
        dV = out[1].view(bs * KVH, skv, D)
    ops = []
    for r in range(1, world):
        u0, u1 = rng(r)
        h0, h1 = head_slice(u0, u1)
        ops.append(dist.P2POp(dist.irecv, dS[h0:h1], r, group))
        ops.append(dist.P2POp(dist.irecv, dV[u0:u1], r, group))
    works = dist.batch_isend_irecv(ops) if ops else []
    u0, u1 = rng(0)
    h0, h1 = head_slice(u0, u1)
    dS[h0:h1].copy_(dS_shard)
    dV[u0:u1].copy_(dV_shard)
    for w in works:
        w.wait()
    return dS.view(bs, H, sq, skv), dV.view(bs, KVH, skv, D)
