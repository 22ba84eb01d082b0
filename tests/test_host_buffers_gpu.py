"""Host-buffer call (C-ABI attn_bwd_b200_host_shard): inputs and outputs in host memory,
copies pipelined against the kernels.  Its results must equal the device call's on the
same inputs: chunk boundaries keep every slice 16-byte aligned and the rows' alignment
classes, so the kernels compute the same rows bit for bit."""
import pytest
import torch

import attn_bwd_b200 as ab
from attn_bwd_b200.generate import generate_input

pytestmark = pytest.mark.gpu

SHAPES = [(6, 384, 384), (3, 37, 53), (2, 64, 96), (5, 129, 200)]


def _host(data, pin=True):
    return tuple(t.contiguous().pin_memory() if pin else t.contiguous() for t in data[:5]) + (data[5],)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("chunks", [0, 1, 5, 64])
def test_host_call_equals_device_call(shape, chunks):
    bs, sq, skv = shape
    data = generate_input(bs, sq, skv, seed=11, device="cpu")
    hS, hV = ab.attn_bwd_host(_host(data), chunks=chunks)
    dS, dV = ab.custom_kernel(tuple(t.cuda() if isinstance(t, torch.Tensor) else t for t in data))
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    assert hS.device.type == "cpu" and hV.device.type == "cpu"
    assert torch.equal(hS, dS.cpu()) and torch.equal(hV, dV.cpu())


def test_host_shard_and_reused_work_buffers():
    bs, sq, skv = 4, 77, 91          # ragged rows; unit step 8 keeps slices aligned
    data = generate_input(bs, sq, skv, seed=12, device="cpu")
    dS, dV = ab.custom_kernel(tuple(t.cuda() if isinstance(t, torch.Tensor) else t for t in data))
    dS, dV = dS.cpu(), dV.cpu()
    dO, P, Pd, V, M, p = data
    for u0, u1 in [(8, 24), (0, 32), (16, 16)]:
        sl = lambda t: t.reshape(bs * 80, sq, skv)[u0 * 10:u1 * 10].contiguous().pin_memory()
        shard = (dO.contiguous().pin_memory(), sl(P), sl(Pd), V.contiguous().pin_memory(), sl(M), p)
        work = tuple(torch.empty(tuple(t.shape), dtype=t.dtype, device="cuda") for t in shard[:5]) + (
            torch.empty(((u1 - u0) * 10, sq, skv), dtype=torch.bfloat16, device="cuda"),
            torch.empty((u1 - u0, skv, 128), dtype=torch.bfloat16, device="cuda"))
        for _ in range(2):           # a second call reuses the same device buffers
            hS, hV = ab.attn_bwd_host(shard, u0, u1, work=work, chunks=3)
            assert torch.equal(hS, dS.reshape(bs * 80, sq, skv)[u0 * 10:u1 * 10])
            assert torch.equal(hV, dV.reshape(bs * 8, skv, 128)[u0:u1])
    assert ab.poll_error() == 0


def test_host_call_pageable_memory():
    data = generate_input(2, 64, 96, seed=13, device="cpu")
    hS, hV = ab.attn_bwd_host(_host(data, pin=False))
    dS, dV = ab.custom_kernel(tuple(t.cuda() if isinstance(t, torch.Tensor) else t for t in data))
    assert torch.equal(hS, dS.cpu()) and torch.equal(hV, dV.cpu())


def test_host_call_ordered_on_current_stream():
    data = generate_input(3, 128, 128, seed=14, device="cpu")
    ref = ab.custom_kernel(tuple(t.cuda() if isinstance(t, torch.Tensor) else t for t in data))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        hS, hV = ab.attn_bwd_host(_host(data), synchronize=False)
        s.synchronize()
    assert torch.equal(hS, ref[0].cpu()) and torch.equal(hV, ref[1].cpu())
