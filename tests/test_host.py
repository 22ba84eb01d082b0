"""Host-side logic of the Python shim and the multi-GPU partition (CPU only)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import attn_bwd_b200 as ab
from attn_bwd_b200.generate import generate_input
from attn_bwd_b200.shard import gather_to_rank0, shard_inputs, unit_range
from oracle.attn_bwd_oracle import attn_bwd_reference, attn_bwd_units


def test_cpu_tensors_are_rejected_no_fallback():
    data = generate_input(1, 4, 16, 1)
    with pytest.raises(ValueError, match="CUDA"):
        ab.custom_kernel(data)


def test_bad_tuple_rejected():
    with pytest.raises(ValueError):
        ab.custom_kernel((1, 2, 3))


def test_wrong_heads_rejected():
    dO = torch.zeros(1, 4, 64, 128, dtype=torch.bfloat16)
    V = torch.zeros(1, 8, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="80"):
        ab.custom_kernel((dO, None, None, V, None, 0.1))


def test_unit_range_partition():
    for n in (1, 7, 16, 384):
        for w in (1, 2, 3, 4, 8):
            rs = [unit_range(n, r, w) for r in range(w)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= 1


def test_aligned_unit_range_keeps_slices_16_byte_aligned():
    """With (sq, skv) the split falls on unit_step boundaries: every rank's first head of
    P / mask starts on a 16-element boundary, and the ranges still tile [0, n)."""
    from attn_bwd_b200.shard import unit_step
    for sq, skv in ((640, 640), (301, 467), (7, 29), (1, 1), (3, 5)):
        g = unit_step(sq, skv)
        assert (10 * g * sq * skv) % 16 == 0
        for n in (8, 16, 96, 384):
            for w in (1, 2, 3, 4, 8):
                rs = [unit_range(n, r, w, sq, skv) for r in range(w)]
                assert rs[0][0] == 0 and rs[-1][1] == n
                assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
                for a, _ in rs:
                    assert (a * 10 * sq * skv) % 16 == 0
                sizes = [b - a for a, b in rs]
                assert max(sizes) - min(sizes) <= g


def test_shard_inputs_are_views_of_the_units_heads():
    data = generate_input(2, 4, 16, 3)
    dO, P, Pd, V, M, p = shard_inputs(data, 3, 11)
    assert P.shape == (80, 4, 16)
    assert torch.equal(P[0], data[1][0, 30]) and torch.equal(P[-1], data[1][1, 29])
    assert P.data_ptr() == data[1][0, 30].data_ptr()


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    bs, sq, skv = 2, 8, 23          # ragged rows: the aligned split has 2-unit steps
    data = generate_input(bs, sq, skv, 5)
    u0, u1 = unit_range(bs * 8, rank, world, sq, skv)
    # each rank computes its units with the CPU oracle (stands in for the GPU call)
    res = attn_bwd_units(data, range(u0, u1))
    dS = torch.cat([res[u][0] for u in range(u0, u1)])
    dV = torch.stack([res[u][1] for u in range(u0, u1)])
    out = gather_to_rank0(dS, dV, bs, sq, skv)
    if rank == 0:
        rS, rV = attn_bwd_reference(data)
        result_q.put((torch.equal(out[0], rS), torch.equal(out[1], rV)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_shard_and_gather(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + world
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) == (True, True)
