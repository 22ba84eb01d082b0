"""Failure detection of the multi-rank path on the host (gloo ranks, no GPU).

A rank that dies before the gather must surface as an error on rank 0 within
the process-group timeout, never as a hang."""
import datetime
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from attn_bwd_b200.shard import gather_to_rank0


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    bs, sq, skv = 1, 2, 16          # 8 units, 4 per rank (unit_step 1)
    dS = torch.zeros(40, sq, skv, dtype=torch.bfloat16)
    dV = torch.zeros(4, skv, 128, dtype=torch.bfloat16)
    if rank == 1:
        os._exit(3)                  # dies between steps, before its sends
    try:
        gather_to_rank0(dS, dV, bs, sq, skv)
        q.put("no error")
    except Exception as e:          # noqa: BLE001
        q.put("error: " + type(e).__name__)
    os._exit(0)


def test_dead_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, 29650, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert procs[1].exitcode == 3
    assert q.get(timeout=5).startswith("error")
