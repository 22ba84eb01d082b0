"""Parity of the CUDA path (through the C-ABI) with the CPU oracle.

Tolerance is the reference's own check (eval_modal_attn_bwd.py:173-197):
torch.allclose(ref.float(), out.float(), rtol=1e-2, atol=1e-2) for dS and dV.
"""
import pytest
import torch

import attn_bwd_b200 as ab
from attn_bwd_b200.generate import generate_input, generate_input_lowmem
from golden_io import CASES, load_case
from oracle.attn_bwd_oracle import attn_bwd_reference, attn_bwd_units

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-2

CONFIGS = {  # BASELINE.json configs c0..c4
    "c0": (2, 64, 96), "c1": (6, 384, 384), "c2": (12, 301, 467),
    "c3": (2, 2048, 3072), "c4": (48, 640, 640),
}
# SOL-ExecBench shapes (eval_modal_attn_bwd.py:18-35), sizes only
SOL_SHAPES = [(4, 256, 256), (8, 373, 449), (4, 1024, 2048), (64, 128, 128), (2, 256, 512),
              (32, 691, 773), (8, 128, 128), (32, 512, 512), (4, 211, 293), (8, 256, 256),
              (16, 128, 256), (1, 1024, 1024), (16, 256, 512), (32, 128, 128), (1, 512, 512),
              (1, 4096, 4096)]


def _close(name, ref, out):
    ok = torch.allclose(ref.float(), out.float().cpu(), rtol=RTOL, atol=ATOL)
    if not ok:
        d = (ref.float() - out.float().cpu()).abs()
        raise AssertionError(f"{name} mismatch: max={d.max().item():.4e} mean={d.mean().item():.4e}")


def _to(data, dev):
    return tuple(t.to(dev) if isinstance(t, torch.Tensor) else t for t in data)


def _check_full(data_cpu, dev):
    data = _to(data_cpu, dev)
    dS, dV = ab.custom_kernel(data)
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    rS, rV = attn_bwd_reference(data_cpu)
    assert dS.shape == rS.shape and dV.shape == rV.shape
    assert dS.dtype == torch.bfloat16 and dV.dtype == torch.bfloat16
    _close("grad_attn_scores", rS, dS)
    _close("grad_value_states", rV, dV)


def _check_sampled(data, units):
    """data on the GPU; compares the listed units with the per-unit oracle."""
    dS, dV = ab.custom_kernel(data)
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    ref = attn_bwd_units(data, units)
    for u in units:
        b, kvh = divmod(u, 8)
        _close(f"dS unit {u}", ref[u][0], dS[b, kvh * 10:kvh * 10 + 10])
        _close(f"dV unit {u}", ref[u][1], dV[b, kvh])


@pytest.mark.parametrize("name", CASES)
def test_golden(name, cuda):
    data, rS, rV, _ = load_case(name)
    dS, dV = ab.custom_kernel(_to(data, cuda))
    torch.cuda.synchronize()
    _close("grad_attn_scores", rS, dS)
    _close("grad_value_states", rV, dV)


@pytest.mark.parametrize("cfg", ["c0", "c1"])
def test_config_full_oracle(cfg, cuda):
    bs, sq, skv = CONFIGS[cfg]
    _check_full(generate_input(bs, sq, skv, 1000 + int(cfg[1])), cuda)


@pytest.mark.parametrize("cfg", ["c2", "c3", "c4"])
def test_config_sampled_units(cfg, cuda):
    bs, sq, skv = CONFIGS[cfg]
    data = generate_input_lowmem(bs, sq, skv, 1000 + int(cfg[1]), device=cuda)
    n = bs * 8
    units = sorted({0, 1, 7, n // 2, n - 1})
    _check_sampled(data, units)


@pytest.mark.parametrize("shape", SOL_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_sol_shapes_sampled(shape, cuda):
    bs, sq, skv = shape
    seed = 1001 + SOL_SHAPES.index(shape)
    data = generate_input_lowmem(bs, sq, skv, seed, device=cuda)
    n = bs * 8
    _check_sampled(data, sorted({0, n // 3, n - 1}))


@pytest.mark.parametrize("shape", [(1, 1, 16), (1, 1, 1), (1, 3, 1), (1, 127, 48), (1, 129, 64),
                                   (2, 64, 272), (1, 200, 512), (1, 17, 528), (1, 64, 40),
                                   (1, 33, 1001), (1, 40, 4160), (1, 9, 4103), (2, 130, 1536), (1, 20, 3001)],
                         ids=lambda s: "x".join(map(str, s)))
def test_edge_shapes(shape, cuda):
    bs, sq, skv = shape
    _check_full(generate_input(bs, sq, skv, 77), cuda)


@pytest.mark.parametrize("p", [0.0, 0.3, -0.5])
def test_dropout_values(p, cuda):
    _check_full(generate_input(1, 64, 128, 5, dropout_p=max(p, 0.0))[:5] + (p,), cuda)


def test_empty_seq_q(cuda):
    data = _to(generate_input(1, 0, 32, 3), cuda)
    dS, dV = ab.custom_kernel(data)
    assert dS.shape == (1, 80, 0, 32)
    assert torch.count_nonzero(dV).item() == 0


def test_noncontiguous_inputs(cuda):
    data_cpu = generate_input(1, 32, 64, 9)
    data = list(_to(data_cpu, cuda))
    data[0] = data[0].transpose(1, 2).contiguous().transpose(1, 2)    # same values, other strides
    dS, dV = ab.custom_kernel(tuple(data))
    rS, rV = attn_bwd_reference(data_cpu)
    _close("dS", rS, dS)
    _close("dV", rV, dV)


def test_repeat_calls_deterministic(cuda):
    data = _to(generate_input(2, 130, 192, 4), cuda)
    a = ab.custom_kernel(data)
    b = ab.custom_kernel(data)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("shape", [(2, 96, 128), (2, 96, 467), (3, 50, 333)])
def test_shard_calls_match_full(shape, cuda):
    """Sharded calls over (batch, kv-head) unit ranges reproduce the full call."""
    bs, sq, skv = shape
    data = _to(generate_input(bs, sq, skv, 21), cuda)
    dS, dV = ab.custom_kernel(data)
    dO, P, Pd, V, M, p = data
    for u0, u1 in [(0, 3), (3, 11), (11, 16)]:
        h0, h1 = u0 * 10, u1 * 10
        sl = lambda t: t.reshape(bs * 80, sq, skv)[h0:h1]
        sS, sV = ab.attn_bwd_shard((dO, sl(P), sl(Pd), V, sl(M), p), u0, u1)
        if (h0 * sq * skv * 2) % 16 == 0:
            # same row alignment as in the full call: same summation order, same bits
            assert torch.equal(sS, dS.reshape(bs * 80, sq, skv)[h0:h1])
        else:
            # the shard is re-based by a copy; rows of seq_kv % 8 != 0 then shift their
            # chunk windows differently (rounding-level differences only)
            _close("shard dS", dS.reshape(bs * 80, sq, skv)[h0:h1].cpu(), sS)
        assert torch.equal(sV, dV.reshape(bs * 8, skv, 128)[u0:u1])


def test_current_stream_ordering(cuda):
    data = _to(generate_input(1, 256, 256, 6), cuda)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        dS, dV = ab.custom_kernel(data)
    s.synchronize()
    rS, rV = attn_bwd_reference(_to(data, "cpu"))
    _close("dS", rS, dS)
    _close("dV", rV, dV)


def test_bounded_wait_reports_and_recovers(cuda):
    """A kernel wait that can never complete gives up after its limit, the error
    is reported through the C-ABI, and the next real call still works."""
    import ctypes
    from attn_bwd_b200 import _lib
    assert ab.poll_error() == 0
    _lib.call("attn_bwd_b200_selftest_wait_timeout", 20000,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert ab.poll_error() == 0x7001
    assert ab.poll_error() == 0          # cleared by the poll
    _check_full(generate_input(1, 16, 64, 8), cuda)


@pytest.mark.parametrize("rows", ["class", "ragged"])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_every_ds_mode(mode, rows, cuda):
    """Each pass-2 mode of the dS kernel (recompute / resident / TMEM-held P / compact), forced
    through the library's test options where the shape allows it, aligned rows and both
    kernels for rows that are not 16-byte multiples (class tiles / per-row re-aligning), with
    and without clusters, against the oracle."""
    shapes = [(1, 100, 192), (1, 70, 640), (1, 40, 1280), (1, 33, 467), (1, 21, 901), (1, 17, 3001),
              (2, 7, 29), (1, 205, 333)]
    bad = []
    with ab.options(ds_mode=mode, row_kind=2 if rows == "class" else 1):
        for shape in shapes:
            data = generate_input(*shape, seed=31)
            dS, dV = ab.custom_kernel(_to(data, cuda))
            torch.cuda.synchronize()
            rS, rV = attn_bwd_reference(data)
            ok = (torch.allclose(rS.float(), dS.float().cpu(), rtol=RTOL, atol=ATOL) and
                  torch.allclose(rV.float(), dV.float().cpu(), rtol=RTOL, atol=ATOL) and ab.poll_error() == 0)
            if not ok:
                bad.append(shape)
    assert not bad, f"mode {mode} rows {rows}: mismatch on {bad}"


def test_release_then_call_again(cuda):
    """Releasing the library's per-device streams, events and cached graphs leaves it usable."""
    data_cpu = generate_input(1, 96, 192, 46)
    data = _to(data_cpu, cuda)
    for _ in range(3):           # eager, captured, replayed
        ab.custom_kernel(data)
    ab.release()
    dS, dV = ab.custom_kernel(data)
    torch.cuda.synchronize()
    rS, rV = attn_bwd_reference(data_cpu)
    _close("dS after release", rS, dS)
    _close("dV after release", rV, dV)


def test_replayed_calls_follow_input_contents(cuda):
    """Repeated full calls on the same buffers are replayed from a cached launch graph; the
    results must follow new input values written into those buffers, and must stay right
    after more distinct argument lists than the cache holds have pushed the entry out."""
    data = list(_to(generate_input(1, 96, 192, 40), cuda))
    out = (torch.empty_like(data[1]), torch.empty_like(data[3]))
    for seed in (41, 42, 43, 44):
        new = generate_input(1, 96, 192, seed)
        for i in range(5):
            data[i].copy_(new[i])
        ab.attn_bwd(tuple(data), out=out)
        torch.cuda.synchronize()
        rS, rV = attn_bwd_reference(new)
        _close(f"dS seed {seed}", rS, out[0])
        _close(f"dV seed {seed}", rV, out[1])
    for skv in range(64, 64 + 24 * 16, 16):       # 24 other argument lists, each seen twice
        small = _to(generate_input(1, 16, skv, 50), cuda)
        ab.custom_kernel(small)
        ab.custom_kernel(small)
    new = generate_input(1, 96, 192, 45)
    for i in range(5):
        data[i].copy_(new[i])
    ab.attn_bwd(tuple(data), out=out)
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    rS, rV = attn_bwd_reference(new)
    _close("dS after eviction", rS, out[0])
    _close("dV after eviction", rV, out[1])


def test_call_inside_caller_graph_capture(cuda):
    """A full call captured into the caller's own CUDA graph replays correctly."""
    data = _to(generate_input(1, 64, 128, 60), cuda)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            ab.custom_kernel(data)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dS, dV = ab.custom_kernel(data)
    new = generate_input(1, 64, 128, 61)
    for i in range(5):
        data[i].copy_(new[i].to(cuda))
    g.replay()
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    rS, rV = attn_bwd_reference(new)
    _close("dS", rS, dS)
    _close("dV", rV, dV)


@pytest.mark.parametrize("shape", [(8, 128, 128), (4, 256, 256), (1, 512, 512), (2, 96, 467)])
def test_repeated_calls_stress(shape, cuda):
    """Hundreds of back-to-back full calls into NaN-filled outputs must all equal the first
    result bit for bit (catches stage-reuse races that corrupt a few rows in rare calls)."""
    bs, sq, skv = shape
    data = _to(generate_input(bs, sq, skv, 70), cuda)
    rS, rV = ab.custom_kernel(data)
    out = (torch.empty_like(rS), torch.empty_like(rV))
    bad = 0
    for _ in range(400):
        out[0].fill_(float("nan"))
        out[1].fill_(float("nan"))
        ab.attn_bwd(data, out=out)
        bad += int(not (torch.equal(out[0], rS) and torch.equal(out[1], rV)))
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    assert bad == 0, f"{bad} of 400 calls differed"
