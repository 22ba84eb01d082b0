"""Benchmark of the B200 attention-backward path (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config c4]

One step = one attention-backward call (fused dS kernel + fused dV kernel) over
this rank's shard of the workload, inputs resident in HBM.  The workload is a
BASELINE config (default c4: bs=48, seq_q=seq_kv=640, 80/8 heads, d=128,
p=0.1), partitioned over ranks by (batch, kv-head) unit with no collective in
the data path (strong scaling: total work fixed).  Between timed steps L2 is
flushed by writing a 256 MiB buffer (as eval_modal_attn_bwd.py:228-231 does).

value = algorithmic bytes of the whole job / max-over-ranks device time, in
GB/s; algorithmic bytes = 7·E + |dO| + 2·|V| (P, P_drop, dS at 2 B, mask at
1 B per score element E = bs·80·sq·skv).

--impl reference times the reference's CPU implementation (the oracle
restatement of attn_bwd/starting_point.py:27-70) on the host cores, on rank 0.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "sol-1-advisor-token-fix_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "attn-bwd µs per call and achieved HBM GB/s (% of roofline) at 1/2/4/8 B200"
CONFIGS = {"c0": (2, 64, 96), "c1": (6, 384, 384), "c2": (12, 301, 467),
           "c3": (2, 2048, 3072), "c4": (48, 640, 640),
           # profiling stand-in: 4 of c4's 48 batch rows (same kernel mode, ~1 GB), so that
           # an ncu capture stays small; its DRAM traffic scales to c4 by 48/4
           "c4s": (4, 640, 640),
           # profiling stand-in for c3: same row length, hence the same cluster form (6 CTAs per
           # row, dP~ resident), a quarter of its rows (~0.9 GB)
           "c3s": (1, 1024, 3072)}
H, KVH, G, D = 80, 8, 10, 128
FALLBACK_HBM_GBS = 6650.0
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one dS-kernel launch per
# (batch, kv-head) unit, from the ncu --set full capture of `bench.py --config c4s --once`
# (c4s = 4 of c4's 48 batch rows, same kernel mode; 669.30 MB over 32 units), scaled by the
# units a launch processes.  Only used for the c4 workload's roofline line.
DS_TRAFFIC_PER_UNIT = {"c4": 669.298e6 / 32}


def alg_bytes(units, sq, skv):
    """Algorithmic (minimum unique) HBM bytes for `units` (batch, kv-head) units."""
    E = units * G * sq * skv
    dO = units * G * sq * D * 2
    V = units * skv * D * 2
    return {"total": 7 * E + dO + 2 * V, "ds": 5 * E + dO + V, "dv": 2 * E + dO + V, "E": E}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def shard_range(n_units, rank, world, sq, skv):
    from attn_bwd_b200.shard import unit_range
    return unit_range(n_units, rank, world, sq, skv)


def _generate_module():
    """attn_bwd_b200/generate.py loaded by file path: the input generator without the
    package (whose import maps the CUDA library), for the CPU-only reference arm."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "_attn_bwd_generate", os.path.join(PKG_DIR, "attn_bwd_b200", "generate.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_shard_inputs(bs, sq, skv, u0, u1, seed, device):
    """Full dO and V, and P / P_drop / mask for heads of units [u0, u1) only.  Batch row b
    is drawn on `device` with seed seed*1000 + b."""
    generate_input = _generate_module().generate_input
    nh = (u1 - u0) * G
    dO = torch.empty(bs, sq, H, D, dtype=torch.bfloat16, device=device)
    V = torch.empty(bs, KVH, skv, D, dtype=torch.bfloat16, device=device)
    P = torch.empty(nh, sq, skv, dtype=torch.bfloat16, device=device)
    Pd = torch.empty_like(P)
    M = torch.empty(nh, sq, skv, dtype=torch.bool, device=device)
    h_lo, h_hi = u0 * G, u1 * G
    for b in range(bs):
        d_b, p_b, pd_b, v_b, m_b, p = generate_input(1, sq, skv, seed * 1000 + b, device=device)
        dO[b].copy_(d_b[0])
        V[b].copy_(v_b[0])
        lo, hi = max(h_lo, b * H), min(h_hi, (b + 1) * H)
        if lo < hi:
            P[lo - h_lo:hi - h_lo].copy_(p_b[0, lo - b * H:hi - b * H])
            Pd[lo - h_lo:hi - h_lo].copy_(pd_b[0, lo - b * H:hi - b * H])
            M[lo - h_lo:hi - h_lo].copy_(m_b[0, lo - b * H:hi - b * H])
        del d_b, p_b, pd_b, v_b, m_b
    return dO, P, Pd, V, M, 0.1


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in the background."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = str(gpu_index)
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", self.idx], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        self.windows = []

    def mark(self, t0, t1):
        self.windows.append((t0, t1))

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.count(",") >= 9]
        os.unlink(self.f.name)
        sm, mx, reasons = [], [], set()
        for r in rows:
            try:
                ts = time.mktime(time.strptime(r[0].split(".")[0], "%Y/%m/%d %H:%M:%S")) + \
                    float("0." + r[0].split(".")[1]) if "." in r[0] else 0.0
            except Exception:
                ts = None
            if ts is not None and self.windows and not any(a - 0.15 <= ts <= b + 0.15 for a, b in self.windows):
                continue
            try:
                sm.append(float(r[2]))
                mx.append(float(r[3]))
            except ValueError:
                continue
            for name, col in (("hw_slowdown", 6), ("hw_thermal_slowdown", 7), ("sw_thermal_slowdown", 8),
                              ("sw_power_cap", 9)):
                if r[col].strip() == "Active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def timed_loop(fn, steps, flush, stream):
    """Per-step CUDA-event times (ms) on the launching stream, L2 flushed between steps."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.fill_(i)
        evs[i][0].record(stream)
        fn()
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.item()


def unit_inputs(cfg, n_units_max=8):
    """CPU copies of the bench workload's own first (batch, kv-head) units: batch row 0 of
    the config drawn exactly as the GPU arm draws it (make_shard_inputs: seed
    (1000 + config index) * 1000, on the GPU when there is one), cut into per-unit tuples
    of the reference layout (10 heads each)."""
    gen = _generate_module()
    bs, sq, skv = CONFIGS[cfg]
    seed = (1000 + int(cfg[1])) * 1000
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    d = gen.generate_input(1, sq, skv, seed, device=dev)
    d = tuple(t.cpu() if isinstance(t, torch.Tensor) else t for t in d)
    units = []
    for kvh in range(min(KVH, n_units_max)):
        hs = slice(kvh * G, kvh * G + G)
        units.append((d[0][:, :, hs].contiguous(), d[1][:, hs].contiguous(), d[2][:, hs].contiguous(),
                      d[3][:, kvh:kvh + 1].contiguous(), d[4][:, hs].contiguous(), d[5]))
    return units, dev


def cpu_sample(cfg, units_target_s=12.0, max_units=100000):
    """Times the CPU oracle on whole (batch, kv-head) units of the config's own inputs until
    about `units_target_s` seconds have passed.  Returns (GB/s, units, seconds)."""
    from oracle.attn_bwd_oracle import _attn_bwd_group
    bs, sq, skv = CONFIGS[cfg]
    torch.set_num_threads(os.cpu_count() or 1)
    units, _ = unit_inputs(cfg)
    _attn_bwd_group(units[0])  # warm-up
    n, t_total = 0, 0.0
    while t_total < units_target_s and n < max_units:
        t0 = time.perf_counter()
        _attn_bwd_group(units[n % len(units)])
        t_total += time.perf_counter() - t0
        n += 1
    gbs = alg_bytes(n, sq, skv)["total"] / t_total / 1e9
    return gbs, n, t_total


def run_reference(args):
    """The reference's CPU implementation of the path (the oracle restatement of
    starting_point.py:27-70; PyTorch fp32 on all host threads) on whole (batch, kv-head)
    units of the config's own inputs.  Loads neither the package nor its CUDA library."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    bs, sq, skv = CONFIGS[args.config]
    from oracle.attn_bwd_oracle import _attn_bwd_group
    torch.set_num_threads(os.cpu_count() or 1)
    units, gen_dev = unit_inputs(args.config)
    units_per_step = 2
    k = 0
    for _ in range(args.warmup):
        for _u in range(units_per_step):
            _attn_bwd_group(units[k % len(units)])
            k += 1
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _u in range(units_per_step):
            _attn_bwd_group(units[k % len(units)])
            k += 1
        times.append(time.perf_counter() - t0)
    t = sum(times)
    gbs = alg_bytes(units_per_step * args.steps, sq, skv)["total"] / t / 1e9
    n_units = bs * KVH
    us_call = (t / (units_per_step * args.steps)) * n_units * 1e6
    cores = torch.get_num_threads()
    sample = (f"{units_per_step} of {n_units} (batch, kv-head) units of {args.config} per step, cycling over "
              f"units 0-{len(units) - 1} of the bench's own seeded inputs (batch row 0, drawn on {gen_dev})")
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t / args.steps * 1e3, 3), "us_per_call": round(us_call, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, eval_modal_attn_bwd.py:139-169 distribution)",
            "config": {"workload": f"{args.config}: bs={bs} seq_q={sq} seq_kv={skv} heads=80/8 d=128 p=0.1",
                       "sample": sample},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


SOL_SHAPES = [(4, 256, 256), (8, 373, 449), (4, 1024, 2048), (64, 128, 128), (2, 256, 512),
              (32, 691, 773), (8, 128, 128), (32, 512, 512), (4, 211, 293), (8, 256, 256),
              (16, 128, 256), (1, 1024, 1024), (16, 256, 512), (32, 128, 128), (1, 512, 512),
              (1, 4096, 4096)]


def _time_like_evaluator(fn, data, flush, reps, warmup):
    """eval_modal_attn_bwd.py:365-401: warm-up calls, then per rep an L2 flush, a
    synchronize and CUDA events around the call (host time of the call counts)."""
    for _ in range(max(warmup, 3)):
        fn(data)
    torch.cuda.synchronize()
    ms = []
    for _ in range(reps):
        flush.fill_(42)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn(data)
        e1.record()
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    return sum(ms) / len(ms) * 1e3


def _load_snapshot(path):
    """A reference submission file loaded the way the evaluator loads one
    (eval_modal_attn_bwd.py:238-247): importlib from its path, module name "submission"."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("submission", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.custom_kernel


def run_sol_sweep(args):
    """The 16 SOL-ExecBench shapes (eval_modal_attn_bwd.py:18-35, sizes only), each timed
    the way the reference evaluator does (eval_modal_attn_bwd.py:365-401).  With
    --snapshot PATH the reference submission at PATH (unmodified) is timed the same way on
    the same GPU and inputs, alternating with this library shape by shape, and its outputs
    are compared with ours (allclose at the evaluator's 1e-2).  Prints one JSON line with
    per-shape us, both geomeans, the per-shape ratio and the reference's score
    756/geomean (eval_modal_attn_bwd.py:417-420)."""
    import math
    import attn_bwd_b200 as ab
    from attn_bwd_b200.generate import generate_input_lowmem
    torch.cuda.set_device(0)
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device="cuda")
    snap = _load_snapshot(args.snapshot) if args.snapshot else None
    rows = []
    for i, (bs, sq, skv) in enumerate(SOL_SHAPES):
        data = generate_input_lowmem(bs, sq, skv, 1001 + i, device="cuda")
        us = _time_like_evaluator(ab.custom_kernel, data, flush, args.steps, args.warmup)
        gbs = alg_bytes(bs * KVH, sq, skv)["total"] / (us * 1e-6) / 1e9
        row = {"bs": bs, "sq": sq, "skv": skv, "us": round(us, 2), "GBps": round(gbs, 1)}
        if snap is not None:
            with torch.no_grad():
                us_ref = _time_like_evaluator(snap, data, flush, args.steps, args.warmup)
                rS, rV = snap(data)
            oS, oV = ab.custom_kernel(data)
            torch.cuda.synchronize()
            row["snapshot_us"] = round(us_ref, 2)
            row["speedup"] = round(us_ref / us, 3)
            row["outputs_match"] = bool(torch.allclose(rS.float(), oS.float(), rtol=1e-2, atol=1e-2) and
                                        torch.allclose(rV.float(), oV.float(), rtol=1e-2, atol=1e-2))
            del rS, rV, oS, oV
        rows.append(row)
        del data
        torch.cuda.empty_cache()
    assert ab.poll_error() == 0
    geo = lambda k: math.exp(sum(math.log(r[k]) for r in rows) / len(rows))
    line = {"sweep": "sol-execbench-16", "geomean_us": round(geo("us"), 2), "score": round(756.0 / geo("us"), 3),
            "reference_best_snapshot_recorded_geomean_us": 379.11, "steps": args.steps, "shapes": rows}
    if snap is not None:
        line["snapshot"] = os.path.basename(args.snapshot)
        line["snapshot_geomean_us_same_gpu"] = round(geo("snapshot_us"), 2)
        line["snapshot_score_same_gpu"] = round(756.0 / geo("snapshot_us"), 3)
        line["geomean_speedup"] = round(geo("snapshot_us") / geo("us"), 3)
    print(json.dumps(line), flush=True)


def run_once(args):
    """Two warm-up rounds then one dS-kernel and one dV-kernel launch on the config."""
    import attn_bwd_b200 as ab
    from attn_bwd_b200.generate import generate_input_lowmem
    bs, sq, skv = CONFIGS[args.config]
    dO, P, Pd, V, M, p = generate_input_lowmem(bs, sq, skv, 7, device="cuda")
    for _ in range(3):
        ab.ds_shard(dO, P, V, M, p, 0, bs * KVH)
        ab.dv_shard(dO, Pd, V, 0, bs * KVH)
    torch.cuda.synchronize()
    assert ab.poll_error() == 0
    print(json.dumps({"once": args.config, "ok": True}))


class NvmlClock:
    """SM clock read through NVML every ~2 ms on a background thread (read-only)."""

    def __init__(self, device_index):
        import threading
        self.samples = []
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._read = lambda: pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._read()
            self.ok = True
        except Exception:
            return
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                self.samples.append((time.perf_counter(), self._read()))
                time.sleep(0.002)
        self._t = threading.Thread(target=loop, daemon=True)
        self._t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self._t.join()

    def during(self, t0, t1):
        """Median SM MHz sampled in [t0, t1], else the sample nearest the interval's middle."""
        xs = [m for t, m in self.samples if t0 <= t <= t1]
        if xs:
            return statistics.median(xs)
        if not self.samples:
            return None
        mid = 0.5 * (t0 + t1)
        return min(self.samples, key=lambda s: abs(s[0] - mid))[1]


def clock_binned(fn, launches, flush, stream, device_index, max_mhz):
    """Each launch timed with CUDA events on its own (synchronised before and after), with
    the SM clock NVML saw during it: launches binned by clock, and each launch's time scaled
    to the maximum clock (us x MHz / max MHz; constant if the kernel's time is set by the
    SM clock, the raw time constant if it is set by HBM)."""
    clk = NvmlClock(device_index)
    rows = []
    for i in range(launches):
        flush.fill_(i)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        t1 = time.perf_counter()
        rows.append((e0.elapsed_time(e1) * 1e3, t0, t1))
    clk.stop()
    if not clk.ok:
        return {"nvml": False, "us_median": round(statistics.median(r[0] for r in rows), 2)}
    per = [(us, clk.during(t0, t1)) for us, t0, t1 in rows]
    per = [(us, m) for us, m in per if m]
    bins = {}
    for us, m in per:
        bins.setdefault(int(round(m / 15.0) * 15), []).append(us)
    mx = max_mhz or max(m for _, m in per)
    return {"nvml": True, "launches": len(per),
            "us_median": round(statistics.median(us for us, _ in per), 2),
            "us_min": round(min(us for us, _ in per), 2), "us_max": round(max(us for us, _ in per), 2),
            "sm_mhz_median": statistics.median(m for _, m in per),
            "us_scaled_to_max_clock_median": round(statistics.median(us * m / mx for us, m in per), 2),
            "bins": {str(k): {"n": len(v), "us_median": round(statistics.median(v), 2)}
                     for k, v in sorted(bins.items())}}


def config_leg(ab, cfg, dev, steps, flush, stream, peak):
    """Whole call, dS kernel alone and dV kernel alone on one more BASELINE config (one
    GPU, all units), timed like the main leg; fractions of the measured HBM peak follow
    from the algorithmic bytes and the printed us."""
    bs, sq, skv = CONFIGS[cfg]
    n = bs * KVH
    data = make_shard_inputs(bs, sq, skv, 0, n, 1000 + int(cfg[1]), dev)
    dO, P, Pd, V, M, p = data
    step = lambda: ab.attn_bwd_shard(data, 0, n)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    call_ms = timed_loop(step, steps, flush, stream)
    ds_ms = timed_loop(lambda: ab.ds_shard(dO, P, V, M, p, 0, n), steps, flush, stream)
    dv_ms = timed_loop(lambda: ab.dv_shard(dO, Pd, V, 0, n), steps, flush, stream)
    assert ab.poll_error() == 0
    b = alg_bytes(n, sq, skv)
    us = lambda ms: sum(ms) / len(ms) * 1e3
    out = {"shape": [bs, sq, skv], "alg_bytes": {"call": b["total"], "ds": b["ds"], "dv": b["dv"]}}
    for name, ms, key in (("call", call_ms, "total"), ("ds_kernel", ds_ms, "ds"), ("dv_kernel", dv_ms, "dv")):
        t = us(ms)
        gbs = b[key] / (t * 1e-6) / 1e9
        out[name] = {"us": round(t, 2), "GBps": round(gbs, 1), "frac": round(gbs / peak, 4)}
    del data, dO, P, Pd, V, M
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS))
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-chunks", type=int, default=0, help="pipeline depth of the host-buffer call (0 = 16)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--once", action="store_true",
                    help="one dS-kernel and one dV-kernel call on the config (for ncu), then exit")
    ap.add_argument("--sweep", choices=["sol"], default=None,
                    help="time the 16 SOL-ExecBench shapes instead of the driver line")
    ap.add_argument("--snapshot", default=None,
                    help="with --sweep sol: a reference submission file to time alongside (unmodified)")
    ap.add_argument("--no-configs", action="store_true", help="skip the c1-c3 block of the line")
    ap.add_argument("--clock-launches", type=int, default=40,
                    help="dS launches timed one by one against the NVML SM clock (0: skip)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.sweep == "sol":
        return run_sol_sweep(args)
    if args.once:
        return run_once(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
    import attn_bwd_b200 as ab

    bs, sq, skv = CONFIGS[args.config]
    n_units = bs * KVH
    u0, u1 = shard_range(n_units, rank, world, sq, skv)
    dev = torch.device("cuda", local)
    data = make_shard_inputs(bs, sq, skv, u0, u1, 1000 + int(args.config[1]), dev)
    dO, P, Pd, V, M, p = data
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        return ab.attn_bwd_shard(data, u0, u1)

    def ds_only():
        return ab.ds_shard(dO, P, V, M, p, u0, u1)

    def dv_only():
        return ab.dv_shard(dO, Pd, V, u0, u1)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert ab.poll_error() == 0

    sampler = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else local)
    time.sleep(0.3)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    w0 = time.time()
    step_ms = timed_loop(step, args.steps, flush, stream)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    w1 = time.time()
    ds_ms = timed_loop(ds_only, args.steps, flush, stream)
    dv_ms = timed_loop(dv_only, args.steps, flush, stream)
    w2 = time.time()
    sampler.mark(w0, w2)
    time.sleep(0.25)
    clocks = sampler.stop()
    assert ab.poll_error() == 0

    t_step = max_over_ranks(sum(step_ms) / 1e3, world)          # seconds for K steps, max over ranks
    t_ds = max_over_ranks(sum(ds_ms) / args.steps / 1e3, world)  # seconds per launch
    t_dv = max_over_ranks(sum(dv_ms) / args.steps / 1e3, world)
    job = alg_bytes(n_units, sq, skv)
    mine = alg_bytes(u1 - u0, sq, skv)
    value = job["total"] * args.steps / t_step / 1e9
    peak, peak_kind = peaks()
    ds_gbs = mine["ds"] / t_ds / 1e9
    dv_gbs = mine["dv"] / t_dv / 1e9

    # ---- end to end through the public API with host buffers (pinned), copies timed:
    # attn_bwd_host pipelines chunks of units over H2D copies, kernels and D2H copies
    host = [t.cpu().pin_memory() for t in (dO, P, Pd, V, M)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    dS_h = torch.empty((u1 - u0) * G, sq, skv, dtype=torch.bfloat16).pin_memory()
    dV_h = torch.empty(u1 - u0, skv, D, dtype=torch.bfloat16).pin_memory()
    d2h = dS_h.numel() * 2 + dV_h.numel() * 2
    work = tuple(torch.empty_like(t, device=dev) for t in host) + (
        torch.empty_like(dS_h, device=dev), torch.empty_like(dV_h, device=dev))
    host_data = tuple(host) + (p,)

    def e2e_step():
        ab.attn_bwd_host(host_data, u0, u1, work=work, out=(dS_h, dV_h), chunks=args.e2e_chunks,
                         synchronize=False)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e2e_ms = timed_loop(e2e_step, args.e2e_steps, flush, stream)
    t_e2e = max_over_ranks(sum(e2e_ms) / 1e3, world)
    e2e_val = job["total"] * args.e2e_steps / t_e2e / 1e9
    # the host-buffer results are the device call's (checked outside the timed region)
    s_, v_ = step()
    torch.cuda.synchronize()
    assert torch.equal(dV_h, v_.cpu()) and torch.equal(dS_h[:2 * G], s_[:2 * G].cpu()), "host-buffer call mismatch"
    del s_, v_

    # ---- gather of every rank's dS / dV shard to rank 0 (NCCL point-to-point), timed
    # separately: it is not part of the per-call kernel time the value reports
    gather_ms = None
    if world > 1:
        from attn_bwd_b200.shard import gather_to_rank0
        s_, v_ = step()
        gather_to_rank0(s_, v_, bs, sq, skv)   # warm-up: NCCL sets up its P2P channels lazily
        torch.cuda.synchronize()
        torch.distributed.barrier()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record()
        out = gather_to_rank0(s_, v_, bs, sq, skv)
        g1.record()
        torch.cuda.synchronize()
        gather_ms = max_over_ranks(g0.elapsed_time(g1), world)
        del out, s_, v_

    # ---- dS launches one by one against the SM clock (rank 0 of a 1-GPU run)
    ds_clock = None
    if world == 1 and args.clock_launches > 0:
        try:
            mx = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))).get("sm_max_mhz", 0))
        except Exception:
            mx = 0.0
        ds_clock = clock_binned(ds_only, args.clock_launches, flush, stream, local, mx)

    # ---- the other BASELINE configs on one GPU (c4 inputs freed first)
    configs = None
    if world == 1 and args.config == "c4" and not args.no_configs:
        del data, dO, P, Pd, V, M, host, host_data, work, dS_h, dV_h
        torch.cuda.empty_cache()
        configs = {}
        for cfg in ("c1", "c2", "c3"):
            configs[cfg] = config_leg(ab, cfg, dev, args.steps, flush, stream, peak)
        configs["c4"] = {"shape": [bs, sq, skv], "call": {"us": round(t_step / args.steps * 1e6, 2),
                                                           "frac": round(value / peak, 4)},
                         "ds_kernel": {"us": round(t_ds * 1e6, 2), "frac": round(ds_gbs / peak, 4)},
                         "dv_kernel": {"us": round(t_dv * 1e6, 2), "frac": round(dv_gbs / peak, 4)}}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, n, secs = cpu_sample(args.config)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} (batch, kv-head) units of {args.config} ({n}/{n_units} of the workload), "
                         f"{secs:.1f} s, oracle restatement of starting_point.py on the host CPU"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_step / args.steps * 1e3, 4),
            "us_per_call": round(t_step / args.steps * 1e6, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, eval_modal_attn_bwd.py:139-169 distribution)",
            "config": {"workload": f"{args.config}: bs={bs} seq_q={sq} seq_kv={skv} heads=80/8 d=128 p=0.1",
                       "partition": f"(batch, kv-head) units, {n_units} over {world} rank(s)",
                       "l2": "256 MiB buffer written between timed steps; inputs also exceed L2",
                       "alg_bytes_per_call": job["total"]},
            "roofline": {"bound": "hbm", "kernel": "ds_kernel", "achieved": round(ds_gbs, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(ds_gbs / peak, 4),
                         "traffic": (round(DS_TRAFFIC_PER_UNIT[args.config] * (u1 - u0))
                                     if args.config in DS_TRAFFIC_PER_UNIT else None),
                         "peak_kind": peak_kind,
                         "alg_bytes_per_launch": mine["ds"], "us_per_launch": round(t_ds * 1e6, 2)},
            "kernels": {
                "ds_kernel": {"us": round(t_ds * 1e6, 2), "GBps": round(ds_gbs, 1), "frac": round(ds_gbs / peak, 4)},
                "dv_kernel": {"us": round(t_dv * 1e6, 2), "GBps": round(dv_gbs, 1), "frac": round(dv_gbs / peak, 4)},
            },
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(t_e2e / args.e2e_steps * 1e3, 2)},
            "gpu_launches": 2 * args.steps,
            "gather_to_rank0_ms": None if gather_ms is None else round(gather_ms, 3),
            "gather_to_rank0_GBps": None if gather_ms is None else round(
                (alg_bytes(n_units, sq, skv)["E"] * 2 + n_units * skv * D * 2) * (world - 1) / world
                / (gather_ms * 1e-3) / 1e9, 1),
            "clocks": clocks,
            "ds_kernel_vs_clock": ds_clock,
            "configs": configs,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
