#!/usr/bin/env python3
"""Benchmark of the B200 probe path (one JSON line on stdout, rank 0).

Headline workload: the sharded HBM copy stream — every GPU copies its own
fp32[2^30] (4 GiB) buffer, seeded uniform [-1,1), to a second buffer with
cmb_stream_copy (the reference's kernel_stream_copy, src/mem_global.cu:13-16,
re-targeted to sm_100a).  One step = one copy of the 4 GiB buffer on every
GPU; value = algorithmic bytes (read + write) of all GPUs / max-over-ranks
device time, in GB/s.  Weak scaling: per-GPU work is fixed.

At N=1, rank 0 also runs the other probes of the path once (1 GiB copy and
sum, 512 MiB chase, TMA tile copy, tcgen05 GEMMs) and reports them under
"probes"; at N>1 the NVLink peer-store ring and all-to-all are reported there.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the CPU implementation of the same copy (the
oracle's multi-threaded memcpy, the reference path having no CPU code of its
own) on a bounded sample, on rank 0 only.
"""

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "HBM GB/s & BF16/FP8 TFLOPS per B200 (% of peak); NVLink P2P GB/s at 1/2/4/8 GPU"
UNIT = "GB/s"
SEED = 0x5EED
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------- ranks


class Ranks:
    """Process-group plumbing: one process per GPU, launched by torchrun."""

    def __init__(self, backend: str, timeout_s: float = 120.0):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        if self.world > 1 and not dist.is_initialized():
            import datetime

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            kw = {}
            if backend == "nccl":
                # bind the group to this rank's GPU (no guessing from the rank)
                torch.cuda.set_device(self.local_rank)
                kw["device_id"] = torch.device("cuda", self.local_rank)
            dist.init_process_group(backend=backend,
                                    timeout=datetime.timedelta(seconds=timeout_s), **kw)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        dev = "cuda" if self.backend == "nccl" else "cpu"
        t = self.torch.tensor([x], dtype=self.torch.float64, device=dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if self.world == 1:
            return x
        dev = "cuda" if self.backend == "nccl" else "cpu"
        t = self.torch.tensor([x], dtype=self.torch.float64, device=dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.world > 1 and self.dist.is_initialized():
            self.dist.destroy_process_group()


# ---------------------------------------------------------------- clocks


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 20):
        self.gpu_index, self.period_ms = gpu_index, period_ms
        self.proc, self.file, self.t0 = None, None, None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 f"-i", str(self.gpu_index), f"-lms", str(self.period_ms)],
                stdout=self.file, stderr=subprocess.DEVNULL)
            self.t0 = time.time()
            # nvidia-smi needs a moment before its first sample: wait for it
            # (up to 2 s) so a short timed region is sampled from its start
            while time.time() - self.t0 < 2.0 and os.path.getsize(self.file.name) == 0:
                time.sleep(0.005)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(2 * self.period_ms / 1000.0)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().splitlines() if r.strip()]
        self.file.close()
        os.unlink(self.file.name)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                power.append(float(r[3]))
            except (ValueError, IndexError):
                continue
            for k, name in enumerate(names):
                if len(r) > 5 + k and r[5 + k].strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------- helpers


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
                "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name: str):
    """dram bytes per launch recorded from ncu in profiles/<name>.txt, if any
    (a line `traffic_bytes_per_launch: <int>`)."""
    path = os.path.join(ROOT, "profiles", name + ".txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


def cpu_memcpy_baseline(sample_bytes: int, steps: int, warmup: int) -> dict:
    """Times the oracle's multi-threaded memcpy (the CPU implementation of the
    copy probe) on a bounded sample; GB/s counts read + write bytes."""
    import numpy as np

    import oracle

    orc = oracle.load()
    threads = orc.orc_hw_threads()
    src = np.empty(sample_bytes, np.uint8)
    dst = np.empty(sample_bytes, np.uint8)
    orc.orc_fill_bytes(oracle.ptr(src), sample_bytes, SEED)
    dst.fill(1)  # fault the pages in
    for _ in range(warmup):
        orc.orc_memcpy_mt(oracle.ptr(dst), oracle.ptr(src), sample_bytes, threads)
    total = 0.0
    for _ in range(steps):
        total += orc.orc_memcpy_mt(oracle.ptr(dst), oracle.ptr(src), sample_bytes, threads)
    assert np.array_equal(src[:: 1 << 16], dst[:: 1 << 16])
    gbs = 2.0 * sample_bytes * steps / total / 1e9
    return {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} x memcpy of {sample_bytes >> 20} MiB (oracle, {threads} threads)",
            "seconds": round(total, 4)}


# ---------------------------------------------------------------- our arm


# Result flags of the probes: a check passed when its flag has this value.
CHECK_FLAGS = {"bit_exact": True, "within_1e-2": True, "within_1e-5": True,
               "endpoint_matches_host_walk": True, "landed_bytes_match": True, "status": 0,
               "bit_equal_to_plain_order": True}


def failed_checks(node, path="") -> list:
    """Paths of every probe check in `node` (nested dicts) that failed."""
    bad = []
    if isinstance(node, dict):
        for k, v in node.items():
            p = f"{path}.{k}" if path else k
            if k in CHECK_FLAGS and not isinstance(v, dict):
                if v != CHECK_FLAGS[k]:
                    bad.append(f"{p}={v}")
            else:
                bad += failed_checks(v, p)
    return bad


def run_ours(args) -> int:
    import torch

    import cuda_micro_bench_b200 as cmbpkg
    from cuda_micro_bench_b200 import check, lib

    ranks = Ranks("nccl")
    torch.cuda.set_device(ranks.local_rank)
    dev_index = torch.cuda.current_device()
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    n = int(args.gib * (1 << 28))
    nbytes = 4 * n
    src = torch.empty(n, dtype=torch.float32, device="cuda")
    dst = torch.empty(n, dtype=torch.float32, device="cuda")
    check("cmb_fill_uniform_f32", ctypes.c_void_p(src.data_ptr()), n,
          ctypes.c_uint64(SEED + ranks.rank), sh)
    dst.zero_()
    torch.cuda.synchronize()

    def step():
        check("cmb_stream_copy", ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src.data_ptr()),
              nbytes, sh)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # correctness of what is being timed: bit-exact copy
    ok = bool(torch.equal(src.view(torch.int32), dst.view(torch.int32)))
    if not ok:
        raise SystemExit(f"rank {ranks.rank}: copy output differs from input")

    clocks = ClockSampler(dev_index, period_ms=5).start()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    ranks.barrier()
    torch.cuda.synchronize()
    evs[0].record(stream)
    for k in range(args.steps):
        step()
        evs[k + 1].record(stream)
    torch.cuda.synchronize()
    ranks.barrier()
    clk = clocks.stop()
    launch_ms = [evs[k].elapsed_time(evs[k + 1]) for k in range(args.steps)]
    local_ms = evs[0].elapsed_time(evs[-1])
    total_ms = ranks.max(local_ms)
    value = ranks.world * 2.0 * nbytes * args.steps / (total_ms * 1e-3) / 1e9

    peaks = measured_peaks()
    avg_launch_s = statistics.mean(launch_ms) * 1e-3
    achieved = 2.0 * nbytes / avg_launch_s / 1e9
    traffic = profile_traffic("stream_copy_4gib")
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": traffic, "peak_source": peaks["source"],
                "kernel": "k_stream_copy<32,2>", "algorithmic_bytes_per_launch": 2 * nbytes}

    # end to end through the C ABI with pinned host buffers
    e2e = run_e2e(args, ranks, torch, src, dst, nbytes) if args.e2e_steps > 0 else None

    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ranks.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded uniform [-1,1) fp32, SplitMix64)",
        "config": {"workload": f"stream_copy: fp32[{n}] ({nbytes / 2**30:g} GiB) -> second "
                               "buffer per GPU, sharded, no exchange",
                   "bytes_per_gpu_per_step": 2 * nbytes, "parallelism": f"shard{ranks.world}",
                   "l2": f"inputs larger than L2 ({nbytes / 2**30:g} GiB vs 126 MB)", "impl": "ours"},
        "roofline": roofline, "e2e": e2e, "gpu_launches": args.steps,
        "clocks": clk,
    }
    if ranks.rank == 0 and ranks.world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_memcpy_baseline(1 << 30, 8, 1)
        if not args.no_probes:
            result["cpu_baseline"]["probes"] = cpu_probe_baselines()
    del src, dst
    torch.cuda.empty_cache()
    if not args.no_probes:
        result["probes"] = run_probes(args, ranks, peaks)
    # every rank's probe checks decide the exit code, so a wrong receive or
    # result on any GPU fails the run instead of only flagging it
    bad = failed_checks(result.get("probes", {}))
    any_bad = ranks.sum(float(len(bad))) > 0
    if ranks.rank == 0:
        print(json.dumps(result), flush=True)
    if bad:
        print(f"rank {ranks.rank}: failed checks: {', '.join(bad)}", file=sys.stderr, flush=True)
    ranks.close()
    return 1 if any_bad else 0


def run_e2e(args, ranks, torch, dev_a, dev_b, nbytes):
    """Same metric through cmb_stream_copy_host: pinned host input, H2D, the
    device copy, D2H of the full result, every step."""
    from cuda_micro_bench_b200 import check

    host_src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host_dst = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host_src.copy_(dev_a.view(torch.uint8).cpu())
    chunk = 64 << 20
    steps = max(1, min(args.e2e_steps, args.steps))

    def e2e_step():
        check("cmb_stream_copy_host", ctypes.c_void_p(host_dst.data_ptr()),
              ctypes.c_void_p(host_src.data_ptr()), nbytes, ctypes.c_void_p(dev_a.data_ptr()),
              ctypes.c_void_p(dev_b.data_ptr()), nbytes, chunk)

    e2e_step()
    if not torch.equal(host_src[:: 1 << 12], host_dst[:: 1 << 12]):
        raise SystemExit("e2e copy output differs from input")
    ranks.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        e2e_step()
    local = time.perf_counter() - t0
    ranks.barrier()
    total = ranks.max(local)
    value = ranks.world * 2.0 * nbytes * steps / total / 1e9
    links = _host_link_rates(torch, ranks, host_src, host_dst, dev_a, dev_b, nbytes)
    del host_src, host_dst
    return {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": nbytes,
            "d2h_bytes_per_step": nbytes, "steps": steps,
            "path": "cmb_stream_copy_host (pinned host -> device copy -> host, 64 MiB chunks)",
            "host_links": links}


def _host_link_rates(torch, ranks, host_src, host_dst, dev_a, dev_b, nbytes) -> dict:
    """What the host side alone carries, all ranks at once: plain pinned
    host->device, device->host and both directions together
    (cudaMemcpyAsync through torch), aggregate GB/s of all ranks from the
    max-over-ranks wall time.  The e2e leg cannot exceed the both-directions
    rate; a rate that grows less than N-fold with N shows a shared host."""
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    d_a, d_b = dev_a.view(torch.uint8), dev_b.view(torch.uint8)

    def h2d():
        d_a.copy_(host_src, non_blocking=True)

    def d2h():
        host_dst.copy_(d_b, non_blocking=True)

    def both():
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            host_dst.copy_(d_b, non_blocking=True)
        d_a.copy_(host_src, non_blocking=True)
        stream.wait_stream(side)

    out = {}
    for name, fn, bytes_moved in (("h2d_GB/s", h2d, nbytes), ("d2h_GB/s", d2h, nbytes),
                                  ("h2d_plus_d2h_GB/s", both, 2 * nbytes)):
        torch.cuda.synchronize()
        ranks.barrier()
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        local = time.perf_counter() - t0
        ranks.barrier()
        out[name] = round(ranks.world * bytes_moved / ranks.max(local) / 1e9, 2)
    out["what"] = (f"{nbytes >> 20} MiB pinned copies per rank, all {ranks.world} ranks at once, "
                   "aggregate")
    return out


# ---------------------------------------------------------------- probes


def _time_launches(torch, stream, fn, reps):
    """Per-launch device times (ms) of `reps` back-to-back calls of fn."""
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    torch.cuda.synchronize()
    evs[0].record(stream)
    for k in range(reps):
        fn()
        evs[k + 1].record(stream)
    torch.cuda.synchronize()
    return [evs[k].elapsed_time(evs[k + 1]) for k in range(reps)]


def _median_ms(torch, stream, fn, reps=9, warm=3):
    """Median device time (ms) of `reps` back-to-back launches after `warm`
    untimed ones (clocks and TLBs settle in the warm-up)."""
    for _ in range(warm):
        fn()
    return statistics.median(_time_launches(torch, stream, fn, reps))


def probe_stream_1gib(torch, stream, sh, peaks):
    """Config: fp32[2^28] (1 GiB) copy (bit-exact) and sum (checked against
    an fp64 sum, rel 1e-5); median of 9 timed launches after 3 warm-up
    launches (the reference's measure() takes the median of 5 after one
    warm-up, src/mem_global.cu:42-53)."""
    from cuda_micro_bench_b200 import check, lib

    n = 1 << 28
    src = torch.empty(n, dtype=torch.float32, device="cuda")
    dst = torch.empty(n, dtype=torch.float32, device="cuda")
    check("cmb_fill_uniform_f32", ctypes.c_void_p(src.data_ptr()), n, ctypes.c_uint64(SEED), sh)
    ws_bytes = lib.cmb_stream_sum_workspace_bytes(n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    copy = lambda: check("cmb_stream_copy", ctypes.c_void_p(dst.data_ptr()),
                         ctypes.c_void_p(src.data_ptr()), 4 * n, sh)
    ssum = lambda: check("cmb_stream_sum_f32", ctypes.c_void_p(src.data_ptr()), n,
                         ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                         ws_bytes, sh)
    copy_ms = _median_ms(torch, stream, copy)
    sum_ms = _median_ms(torch, stream, ssum)
    copy_ok = bool(torch.equal(src.view(torch.int32), dst.view(torch.int32)))
    ref = float(src.double().sum().item())  # fp64 check sum
    got = float(out.item())
    rel = abs(got - ref) / abs(ref)
    copy_gbs = 2.0 * 4 * n / (copy_ms * 1e-3) / 1e9
    read_gbs = 4.0 * n / (sum_ms * 1e-3) / 1e9
    del src, dst, ws, out
    return {
        "copy_1gib": {"GB/s": round(copy_gbs, 2), "frac_of_measured_hbm": round(copy_gbs / peaks["hbm_gbs"], 4),
                      "frac_of_8tbs_spec": round(copy_gbs / 8000.0, 4), "bit_exact": copy_ok,
                      "ms": round(copy_ms, 4)},
        "sum_1gib": {"GB/s": round(read_gbs, 2), "frac_of_measured_hbm": round(read_gbs / peaks["hbm_gbs"], 4),
                     "frac_of_8tbs_spec": round(read_gbs / 8000.0, 4), "sum": got, "fp64_sum": ref,
                     "rel_err": rel, "within_1e-5": rel <= 1e-5, "ms": round(sum_ms, 4)},
    }


def probe_chase(torch, stream, sh, hops):
    """Config: 512 MiB link array, Sattolo cycle from a seed, dependent
    .cg loads; final index vs the host walk (the reference's self-check,
    include/memory_chase.h:152-164)."""
    import numpy as np

    from cuda_micro_bench_b200 import check

    nbytes = 512 << 20
    links = np.empty(nbytes // 4, np.uint32)
    check("cmb_chase_build_links", ctypes.c_void_p(links.ctypes.data), nbytes,
          ctypes.c_uint64(0xC0DA))
    d = torch.from_numpy(links.view(np.int32)).cuda()
    out = torch.zeros(4, dtype=torch.int64, device="cuda")
    warm = 1024
    check("cmb_chase_run", ctypes.c_void_p(d.data_ptr()), links.size, ctypes.c_uint64(warm),
          ctypes.c_uint64(hops), 1, ctypes.c_void_p(out.data_ptr()), sh)
    torch.cuda.synchronize()
    cycles, idx, ns, status = [int(v) for v in out.cpu().numpy().view(np.uint64)]
    expect = ctypes.c_uint32(0)
    check("cmb_chase_host_walk", ctypes.c_void_p(links.ctypes.data), links.size,
          ctypes.c_uint64(warm + hops), ctypes.byref(expect))
    expect = expect.value
    del d
    return {"working_set_bytes": nbytes, "hops": hops, "ns_per_hop": round(ns / hops, 3),
            "cycles_per_hop": round(cycles / hops, 3), "status": status,
            "endpoint_matches_host_walk": idx == expect}


def probe_tma(torch, stream, sh, peaks):
    """Config: 16384 x 16384 bf16 N(0,1), 128x128 boxes, 4-stage mbarrier
    ring, TMA store; bit-exact.  Also the load-only pipeline (the reference's
    tma_g2s_load_bw_gibps) and the 16-byte 1-D TMA round trip."""
    from cuda_micro_bench_b200 import check

    n = 16384
    src = torch.empty(n * n, dtype=torch.int16, device="cuda")
    dst = torch.zeros_like(src)
    check("cmb_fill_normal_bf16", ctypes.c_void_p(src.data_ptr()), n * n, ctypes.c_uint64(SEED),
          ctypes.c_float(1.0), sh)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    xor = torch.zeros(4096, dtype=torch.int32, device="cuda")
    out = {}
    for label, stages, ctas in (("tile_copy_4stage", 4, 1), ("tile_copy_3stage", 3, 1)):
        fn = lambda: check("cmb_tma_tile_copy_bf16", ctypes.c_void_p(dst.data_ptr()),
                           ctypes.c_void_p(src.data_ptr()), n, n, 128, 128, stages, ctas,
                           ctypes.c_void_p(status.data_ptr()), sh)
        ms = _median_ms(torch, stream, fn)
        gbs = 2.0 * 2 * n * n / (ms * 1e-3) / 1e9
        out[label] = {"GB/s": round(gbs, 2), "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                      "frac_of_8tbs_spec": round(gbs / 8000.0, 4), "stages": stages, "box": [128, 128],
                      "bit_exact": bool(torch.equal(src, dst)), "status": int(status.item()),
                      "ms": round(ms, 4)}
    # TMA loads with load/store-unit stores (the stage frees once read into
    # registers), 3 stages x 2 CTAs per SM
    fn = lambda: check("cmb_tma_tile_copy_tuned", ctypes.c_void_p(dst.data_ptr()),
                       ctypes.c_void_p(src.data_ptr()), n, n, 128, 128, 3, 2, 4,
                       ctypes.c_void_p(status.data_ptr()), sh)
    dst.zero_()
    ms = _median_ms(torch, stream, fn)
    gbs = 2.0 * 2 * n * n / (ms * 1e-3) / 1e9
    out["tile_copy_tma_load_lsu_store"] = {
        "GB/s": round(gbs, 2), "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
        "stages": 3, "ctas_per_sm": 2, "box": [128, 128], "bit_exact": bool(torch.equal(src, dst)),
        "status": int(status.item()), "ms": round(ms, 4)}
    fn = lambda: check("cmb_tma_tile_load_bf16", ctypes.c_void_p(src.data_ptr()), n, n, 128, 128,
                       4, ctypes.c_void_p(xor.data_ptr()), 4096,
                       ctypes.c_void_p(status.data_ptr()), sh)
    ms = _median_ms(torch, stream, fn)
    gbs = 2.0 * n * n / (ms * 1e-3) / 1e9
    out["load_only_4stage"] = {"GB/s": round(gbs, 2), "GiB/s": round(gbs / 1.073741824, 2),
                               "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                               "status": int(status.item())}
    buf = torch.empty(1024, dtype=torch.uint8, device="cuda")
    check("cmb_fill_bytes", ctypes.c_void_p(buf.data_ptr()), 1024, ctypes.c_uint64(SEED), sh)
    cyc = torch.zeros(1, dtype=torch.int32, device="cuda")
    landed = torch.zeros(16, dtype=torch.uint8, device="cuda")
    check("cmb_tma_1d_latency", ctypes.c_void_p(buf.data_ptr()), 1024, 0, 256,
          ctypes.c_void_p(cyc.data_ptr()), ctypes.c_void_p(landed.data_ptr()),
          ctypes.c_void_p(status.data_ptr()), sh)
    torch.cuda.synchronize()
    out["tma_1d"] = {"load_latency_cyc": int(cyc.item()) / 256, "round_trips": 256,
                     "landed_bytes_match": bool(torch.equal(landed, buf[:16])),
                     "status": int(status.item())}
    del src, dst
    return out


def install_die_map(sh):
    """Measures the die of every SM (cmb_sm_die_map) and installs the map
    for the GEMMs (cmb_gemm_set_sm_die_map), which then run in the die-split
    tile order.  Returns (labels or None, a summary for the JSON line)."""
    import cuda_micro_bench_b200 as cmbpkg

    t0 = time.perf_counter()
    try:
        labels, near, far = cmbpkg.sm_die_map(sh)
    except cmbpkg.CmbError as e:
        cmbpkg.set_sm_die_map(None)
        return None, {"installed": False, "error": str(e)[:200]}
    ms = (time.perf_counter() - t0) * 1e3
    cmbpkg.set_sm_die_map(labels)
    present = labels[labels != 0xFF]
    return labels, {"installed": True, "sms_on_die": [int((present == d).sum()) for d in (0, 1)],
                    "cold_load_cycles_near_far": [round(near), round(far)],
                    "probe_ms": round(ms, 1)}


def probe_gemm(torch, stream, sh, peaks):
    """Config: M=N=K=8192, A/B bf16 N(0,1)*K^-0.5, fp32 accumulation in
    TMEM, 2-CTA tiles of 256 x 512 (two N=256 accumulators per pair, held
    8-warp epilogue), and the 1-CTA 128x256 form; FP8 e4m3 with a per-tensor
    scale.  The die map is measured and installed first, so the GEMMs run in
    the die-split tile order; the 2-CTA fp32-C forms are also timed in the
    plain order and their outputs compared bit for bit.  TFLOP/s = 2*M*N*K /
    median launch time; every variant's output is checked on 64 sampled
    256x256 tiles (the two corner tiles included) against an fp64 product of
    the same operands (max-norm per tile, rel tol 1e-2).  cuBLAS (torch.mm /
    torch._scaled_mm) on the same operands with the same fp32 output is
    timed alongside as a live reference point; it is not part of the
    product."""
    import cuda_micro_bench_b200 as cmbpkg
    from cuda_micro_bench_b200 import check

    labels, die_summary = install_die_map(sh)

    def plain_order(entry, fn, flop_):
        """Times fn without the die map and compares its C with the die-split C."""
        if labels is None:
            return
        split_c = C.clone()
        cmbpkg.set_sm_die_map(None)
        try:
            ms_ = _median_ms(torch, stream, fn)
            entry["bit_equal_to_plain_order"] = bool(torch.equal(C, split_c))
        finally:
            cmbpkg.set_sm_die_map(labels)
        entry["plain_order_TFLOP/s"] = round(flop_ / (ms_ * 1e-3) / 1e12, 1)
        del split_c

    M = N = K = 8192
    flop = 2.0 * M * N * K
    A = torch.empty(M * K, dtype=torch.int16, device="cuda")
    B = torch.empty(N * K, dtype=torch.int16, device="cuda")
    check("cmb_fill_normal_bf16", ctypes.c_void_p(A.data_ptr()), M * K, ctypes.c_uint64(SEED + 1),
          ctypes.c_float(K ** -0.5), sh)
    check("cmb_fill_normal_bf16", ctypes.c_void_p(B.data_ptr()), N * K, ctypes.c_uint64(SEED + 2),
          ctypes.c_float(K ** -0.5), sh)
    C = torch.empty(M * N, dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    qa = torch.empty(M * K, dtype=torch.uint8, device="cuda")
    qb = torch.empty(N * K, dtype=torch.uint8, device="cuda")
    sa = torch.zeros(2, dtype=torch.float32, device="cuda")
    sb = torch.zeros(2, dtype=torch.float32, device="cuda")
    check("cmb_quantize_e4m3", ctypes.c_void_p(A.data_ptr()), M * K, ctypes.c_void_p(qa.data_ptr()),
          ctypes.c_void_p(sa.data_ptr()), sh)
    check("cmb_quantize_e4m3", ctypes.c_void_p(B.data_ptr()), N * K, ctypes.c_void_p(qb.data_ptr()),
          ctypes.c_void_p(sb.data_ptr()), sh)
    g = torch.Generator().manual_seed(3)
    T = 256  # sampled tile edge
    rows = (torch.randint(0, M // T, (64,), generator=g) * T).tolist()
    cols = (torch.randint(0, N // T, (64,), generator=g) * T).tolist()
    rows[0], cols[0], rows[1], cols[1] = 0, 0, M - T, N - T

    def tiles_err(out, a_f64, b_f64):
        """Max over the sampled tiles of max|C - C_fp64| / max|C_fp64|."""
        Cm = out.view(M, N)
        worst = 0.0
        for r, c in zip(rows, cols):
            ref = a_f64[r:r + T] @ b_f64[c:c + T].T
            got = Cm[r:r + T, c:c + T].double()
            if not bool(torch.isfinite(got).all()):
                return float("inf")
            worst = max(worst, float((got - ref).abs().max() / ref.abs().max()))
        return worst

    sampled_err = lambda a_f64, b_f64: tiles_err(C, a_f64, b_f64)

    a64 = A.view(M, K).view(torch.bfloat16).double()
    b64 = B.view(N, K).view(torch.bfloat16).double()
    out = {"die_map": die_summary}
    for label, cg in (("bf16_8192_2cta", 2), ("bf16_8192_1cta", 1)):
        fn = lambda: check("cmb_gemm_bf16", ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                           ctypes.c_void_p(C.data_ptr()), M, N, K, cg,
                           ctypes.c_void_p(status.data_ptr()), sh)
        ms = _median_ms(torch, stream, fn)
        tf = flop / (ms * 1e-3) / 1e12
        err = sampled_err(a64, b64)
        out[label] = {"TFLOP/s": round(tf, 1), "frac_of_measured_bf16": round(tf / peaks["bf16_tflops"], 4),
                      "frac_of_2250_spec": round(tf / 2250.0, 4), "ms": round(ms, 4),
                      "sampled_tiles_max_rel_err": err, "within_1e-2": err <= 1e-2,
                      "status": int(status.item())}
        if cg == 2:
            plain_order(out[label], fn, flop)
    # the configuration's literal tile: 256 x 256 per 2-CTA pair (one N=256
    # MMA per K slice, two accumulators so the epilogue overlaps)
    fn = lambda: check("cmb_gemm_tuned", ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                       ctypes.c_void_p(C.data_ptr()), M, N, K, 0, None, None, 2, 4, 8, 0, 256, 4,
                       ctypes.c_void_p(status.data_ptr()), sh)
    ms = _median_ms(torch, stream, fn)
    tf = flop / (ms * 1e-3) / 1e12
    err = sampled_err(a64, b64)
    out["bf16_8192_2cta_256x256"] = {
        "TFLOP/s": round(tf, 1), "frac_of_measured_bf16": round(tf / peaks["bf16_tflops"], 4),
        "ms": round(ms, 4), "sampled_tiles_max_rel_err": err, "within_1e-2": err <= 1e-2,
        "status": int(status.item())}
    del a64, b64

    def deq(q, s, rows_, cols_):
        return q.view(rows_, cols_).view(torch.float8_e4m3fn).double() * float(s[0].item())

    a8, b8 = deq(qa, sa, M, K), deq(qb, sb, N, K)
    for label, cg in (("fp8_e4m3_8192_2cta", 2), ("fp8_e4m3_8192_1cta", 1)):
        fn = lambda: check("cmb_gemm_e4m3", ctypes.c_void_p(qa.data_ptr()), ctypes.c_void_p(qb.data_ptr()),
                           ctypes.c_void_p(C.data_ptr()), M, N, K, ctypes.c_void_p(sa.data_ptr()),
                           ctypes.c_void_p(sb.data_ptr()), cg, ctypes.c_void_p(status.data_ptr()), sh)
        ms = _median_ms(torch, stream, fn)
        tf = flop / (ms * 1e-3) / 1e12
        err = sampled_err(a8, b8)
        out[label] = {"TFLOP/s": round(tf, 1), "frac_of_4500_spec": round(tf / 4500.0, 4),
                      "frac_of_2x_measured_bf16": round(tf / (2 * peaks["bf16_tflops"]), 4),
                      "ms": round(ms, 4), "sampled_tiles_max_rel_err": err,
                      "within_1e-2": err <= 1e-2, "status": int(status.item())}
        if cg == 2:
            plain_order(out[label], fn, flop)
    # bf16 C (each fp32 accumulator rounded to nearest even), the output type
    # of the measured bf16 peak: cmb_gemm_bf16_out, 2-CTA held-epilogue tiles
    Cb = torch.empty(M * N, dtype=torch.bfloat16, device="cuda")
    a64 = A.view(M, K).view(torch.bfloat16).double()
    b64 = B.view(N, K).view(torch.bfloat16).double()

    sampled_err_b = lambda a_f64, b_f64: tiles_err(Cb, a_f64, b_f64)

    for label, fp8, ops, scales, (fa, fb) in (
            ("bf16_8192_2cta_bf16out", 0, (A, B), (None, None), (a64, b64)),
            ("fp8_e4m3_8192_2cta_bf16out", 1, (qa, qb),
             (ctypes.c_void_p(sa.data_ptr()), ctypes.c_void_p(sb.data_ptr())), (a8, b8))):
        fn = lambda: check("cmb_gemm_bf16_out", ctypes.c_void_p(ops[0].data_ptr()),
                           ctypes.c_void_p(ops[1].data_ptr()), ctypes.c_void_p(Cb.data_ptr()),
                           M, N, K, fp8, scales[0], scales[1],
                           ctypes.c_void_p(status.data_ptr()), sh)
        ms = _median_ms(torch, stream, fn)
        tf = flop / (ms * 1e-3) / 1e12
        err = sampled_err_b(fa, fb)
        entry = {"TFLOP/s": round(tf, 1), "ms": round(ms, 4), "sampled_tiles_max_rel_err": err,
                 "within_1e-2": err <= 1e-2, "status": int(status.item())}
        if fp8:
            entry["frac_of_4500_spec"] = round(tf / 4500.0, 4)
        else:
            entry["frac_of_measured_bf16"] = round(tf / peaks["bf16_tflops"], 4)
            entry["frac_of_2250_spec"] = round(tf / 2250.0, 4)
        out[label] = entry
    del a8, b8, a64, b64
    # cuBLAS on the same operands, fp32 output like the kernels above
    a16, b16 = A.view(M, K).view(torch.bfloat16), B.view(N, K).view(torch.bfloat16)
    f8a, f8b = qa.view(M, K).view(torch.float8_e4m3fn), qb.view(N, K).view(torch.float8_e4m3fn)
    live = {}
    try:
        ms = _median_ms(torch, stream, lambda: torch.mm(a16, b16.t(), out_dtype=torch.float32))
        live["bf16_TFLOP/s"] = round(flop / (ms * 1e-3) / 1e12, 1)
        ms = _median_ms(torch, stream, lambda: torch._scaled_mm(
            f8a, f8b.t(), scale_a=sa[0], scale_b=sb[0], out_dtype=torch.float32))
        live["e4m3_TFLOP/s"] = round(flop / (ms * 1e-3) / 1e12, 1)
        ms = _median_ms(torch, stream, lambda: torch.mm(a16, b16.t()))
        live["bf16_bf16out_TFLOP/s"] = round(flop / (ms * 1e-3) / 1e12, 1)
        ms = _median_ms(torch, stream, lambda: torch._scaled_mm(
            f8a, f8b.t(), scale_a=sa[0], scale_b=sb[0], out_dtype=torch.bfloat16))
        live["e4m3_bf16out_TFLOP/s"] = round(flop / (ms * 1e-3) / 1e12, 1)
    except (RuntimeError, TypeError) as e:  # an older torch without these forms
        live["error"] = str(e).splitlines()[0][:200]
    if "bf16_TFLOP/s" in live:
        out["bf16_8192_2cta"]["frac_of_live_cublas"] = round(
            out["bf16_8192_2cta"]["TFLOP/s"] / live["bf16_TFLOP/s"], 4)
    if "e4m3_TFLOP/s" in live:
        out["fp8_e4m3_8192_2cta"]["frac_of_live_cublas"] = round(
            out["fp8_e4m3_8192_2cta"]["TFLOP/s"] / live["e4m3_TFLOP/s"], 4)
    for ours, theirs in (("bf16_8192_2cta_bf16out", "bf16_bf16out_TFLOP/s"),
                         ("fp8_e4m3_8192_2cta_bf16out", "e4m3_bf16out_TFLOP/s")):
        if theirs in live:
            out[ours]["frac_of_live_cublas"] = round(out[ours]["TFLOP/s"] / live[theirs], 4)
    live["what"] = ("torch.mm / torch._scaled_mm (cuBLASLt), same operands, fp32 C (and bf16 C "
                    "for the *_bf16out keys), timed alongside")
    out["cublas_same_operands"] = live
    # Back to back for a fixed time with the SM clock sampled: the rate each
    # kernel holds under the power cap, and the rate per GHz of the clock it
    # ran at (the two GEMMs compared at equal clocks).
    dev_index = torch.cuda.current_device()
    ours_bf16 = lambda: check("cmb_gemm_bf16_out", ctypes.c_void_p(A.data_ptr()),
                              ctypes.c_void_p(B.data_ptr()), ctypes.c_void_p(Cb.data_ptr()), M, N, K,
                              0, None, None, ctypes.c_void_p(status.data_ptr()), sh)
    ours_e4m3 = lambda: check("cmb_gemm_bf16_out", ctypes.c_void_p(qa.data_ptr()),
                              ctypes.c_void_p(qb.data_ptr()), ctypes.c_void_p(Cb.data_ptr()), M, N, K,
                              1, ctypes.c_void_p(sa.data_ptr()), ctypes.c_void_p(sb.data_ptr()),
                              ctypes.c_void_p(status.data_ptr()), sh)
    sustained = {}
    try:
        for label, fn in (("ours_bf16_bf16out", ours_bf16),
                          ("cublas_bf16_bf16out", lambda: torch.mm(a16, b16.t())),
                          ("ours_e4m3_bf16out", ours_e4m3),
                          ("cublas_e4m3_bf16out", lambda: torch._scaled_mm(
                              f8a, f8b.t(), scale_a=sa[0], scale_b=sb[0], out_dtype=torch.bfloat16))):
            sustained[label] = _sustained(torch, stream, fn, flop, dev_index)
        if labels is not None:  # ours again in the plain tile order
            cmbpkg.set_sm_die_map(None)
            try:
                for label, fn in (("ours_bf16_bf16out_plain_order", ours_bf16),
                                  ("ours_e4m3_bf16out_plain_order", ours_e4m3)):
                    sustained[label] = _sustained(torch, stream, fn, flop, dev_index)
            finally:
                cmbpkg.set_sm_die_map(labels)
        sustained["what"] = ("each GEMM (8192^3, bf16 C) back to back for ~1 s with nvidia-smi "
                             "sampling the SM clock every 5 ms; ours in the die-split tile order "
                             "and, *_plain_order, without the die map")
    except (RuntimeError, TypeError) as e:
        sustained["error"] = str(e).splitlines()[0][:200]
    out["sustained_with_clocks"] = sustained
    del A, B, C, Cb, qa, qb, a16, b16, f8a, f8b
    return out


def _sustained(torch, stream, fn, flop, dev_index, seconds=1.0):
    """TFLOP/s of fn run back to back for about `seconds` (device time, CUDA
    events), the median SM clock sampled meanwhile, and TFLOP/s per GHz."""
    for _ in range(3):
        fn()
    ms = statistics.median(_time_launches(torch, stream, fn, 5))
    reps = max(10, int(seconds * 1e3 / ms))
    clocks = ClockSampler(dev_index, period_ms=5).start()
    time.sleep(0.05)
    t = _time_launches(torch, stream, fn, reps)
    clk = clocks.stop()
    tf = flop * reps / (sum(t) * 1e-3) / 1e12
    res = {"TFLOP/s": round(tf, 1), "launches": reps, "sm_mhz": clk.get("sm_mhz"),
           "power_w_max": clk.get("power_w_max"), "reasons": clk.get("reasons")}
    if clk.get("sm_mhz"):
        res["TFLOP/s_per_GHz"] = round(tf / (clk["sm_mhz"] / 1e3), 1)
    return res


def _nccl_reference(ranks, nbytes, reps=5, warm=2) -> dict:
    """NCCL over the same links as a live reference point (not the product):
    a ring of send/recv (rank r -> r+1) and all_to_all_single of `nbytes` per
    GPU; per-GPU egress GB/s from the max-over-ranks median time."""
    import torch

    dist = ranks.dist
    stream = torch.cuda.current_stream()
    send = torch.empty(nbytes, dtype=torch.uint8, device="cuda").fill_(ranks.rank & 0xFF)
    recv = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    nxt, prv = (ranks.rank + 1) % ranks.world, (ranks.rank - 1) % ranks.world

    def ring():
        ops = [dist.P2POp(dist.isend, send, nxt), dist.P2POp(dist.irecv, recv, prv)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()

    def a2a():
        dist.all_to_all_single(recv, send)

    out = {}
    for name, fn, egress in (("ring_nccl", ring, nbytes),
                             ("alltoall_nccl", a2a, nbytes * (ranks.world - 1) // ranks.world)):
        times = []
        for rep in range(warm + reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            ranks.barrier()
            torch.cuda.synchronize()
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            t = ranks.max(a.elapsed_time(b))
            if rep >= warm:
                times.append(t)
        ms = statistics.median(times)
        link = egress / (ms * 1e-3) / 1e9
        ok = bool(torch.all(recv[:4096] == (prv if name == "ring_nccl" else 0) & 0xFF))
        out[name] = {"per_gpu_egress_GB/s": round(link, 2), "frac_of_900_spec": round(link / 900.0, 4),
                     "ms": round(ms, 4), "egress_bytes_per_gpu": egress,
                     "received_first_chunk_ok": ok}
    del send, recv
    return out


def probe_p2p(args, ranks) -> dict:
    """Config: 256 MiB seeded random bytes per GPU exchanged over NVLink,
    ring (-> rank+1) and all-to-all (N chunks, each rank visiting its peers
    in staggered order), by in-kernel peer stores, by in-kernel bulk copies,
    by the copy engines (all peers at once, or one or two streams visiting
    them in turn) and by both at once (hybrid_<P>_<S>: the copy engines take
    P/1000 of every job on S streams, peer stores the rest); bit-exact
    receive check.  Time = max over ranks
    of each rank's device time (CUDA events), median of 5 repetitions.  The
    fraction of the peer-copy ceiling divides by the copy engines' ring rate
    measured in the same run; NCCL's send/recv ring and all_to_all_single on
    the same sizes are timed alongside as a reference point."""
    import torch

    from cuda_micro_bench_b200 import multi_gpu

    nbytes = 1 << 28
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    ex = multi_gpu.PeerExchange(ranks, nbytes, SEED)
    out = {}
    methods = {"ring": ("copy_engine", "store", "bulk", "hybrid_700_1"),
               "alltoall": ("store", "bulk", "copy_engine", "copy_engine_1stream",
                            "copy_engine_2stream", "hybrid_500_1")}
    try:
        for mode in ("ring", "alltoall"):
            egress = multi_gpu.egress_bytes(mode, ranks.rank, ranks.world, nbytes)
            for method in methods[mode]:
                times = []
                for rep in range(2 + 5):
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    ranks.barrier()
                    torch.cuda.synchronize()
                    a.record(stream)
                    ex.launch(mode, method, sh)
                    b.record(stream)
                    torch.cuda.synchronize()
                    ranks.barrier()
                    t = ranks.max(a.elapsed_time(b))
                    if rep >= 2:
                        times.append(t)
                ms = statistics.median(times)
                bad = ranks.sum(float(ex.mismatches(mode, sh)))
                link = egress / (ms * 1e-3) / 1e9
                out[f"{mode}_{method}"] = {
                    "per_gpu_egress_GB/s": round(link, 2),
                    "aggregate_GB/s": round(ranks.world * link, 2),
                    "frac_of_900_spec": round(link / 900.0, 4),
                    "ms": round(ms, 4), "egress_bytes_per_gpu": egress,
                    "sm_ctas": {"store": "2 per SM", "bulk": "32 per job (<= SMs / jobs)"}.get(
                        method, "2 per SM and the copy engines" if method.startswith("hybrid")
                        else "0 (copy engines)"),
                    "bit_exact": bad == 0}
        ceiling = out["ring_copy_engine"]["per_gpu_egress_GB/s"]
        for v in out.values():
            v["frac_of_measured_peer_copy"] = round(v["per_gpu_egress_GB/s"] / ceiling, 4)
        out["measured_peer_copy_GB/s"] = {
            "value": ceiling, "what": "copy engines, 256 MiB ring, this run (the denominator of "
                                      "frac_of_measured_peer_copy)"}
    finally:
        ex.close()
    try:
        out["nccl_reference"] = _nccl_reference(ranks, nbytes)
    except (RuntimeError, AttributeError) as e:  # reference point only
        out["nccl_reference"] = {"error": str(e).splitlines()[0][:200]}
    return out


def probe_cublas(torch, stream, sh, ours_tile256=False) -> dict:
    """The live reference of the GEMM probe alone, for profiling it: cuBLAS
    (torch.mm) on the configuration's 8192^3 bf16 operands, fp32 and bf16 C,
    median of 9 launches after 3 warm-up launches each.  With ours_tile256,
    the configuration's literal 2-CTA 256 x 256 tile of this library instead
    (cmb_gemm_tuned, fp32 C)."""
    from cuda_micro_bench_b200 import check

    M = N = K = 8192
    A = torch.empty(M * K, dtype=torch.int16, device="cuda")
    B = torch.empty(N * K, dtype=torch.int16, device="cuda")
    check("cmb_fill_normal_bf16", ctypes.c_void_p(A.data_ptr()), M * K, ctypes.c_uint64(SEED + 1),
          ctypes.c_float(K ** -0.5), sh)
    check("cmb_fill_normal_bf16", ctypes.c_void_p(B.data_ptr()), N * K, ctypes.c_uint64(SEED + 2),
          ctypes.c_float(K ** -0.5), sh)
    a16, b16 = A.view(M, K).view(torch.bfloat16), B.view(N, K).view(torch.bfloat16)
    flop = 2.0 * M * N * K
    out = {}
    if ours_tile256:
        C = torch.empty(M * N, dtype=torch.float32, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        ms = _median_ms(torch, stream, lambda: check(
            "cmb_gemm_tuned", ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
            ctypes.c_void_p(C.data_ptr()), M, N, K, 0, None, None, 2, 4, 8, 0, 256, 4,
            ctypes.c_void_p(status.data_ptr()), sh))
        out["bf16_2cta_256x256_TFLOP/s"] = round(flop / (ms * 1e-3) / 1e12, 1)
        out["status"] = int(status.item())
        return out
    ms = _median_ms(torch, stream, lambda: torch.mm(a16, b16.t(), out_dtype=torch.float32))
    out["bf16_fp32out_TFLOP/s"] = round(flop / (ms * 1e-3) / 1e12, 1)
    ms = _median_ms(torch, stream, lambda: torch.mm(a16, b16.t()))
    out["bf16_bf16out_TFLOP/s"] = round(flop / (ms * 1e-3) / 1e12, 1)
    return out


def probe_gemm_die(torch, stream, sh) -> dict:
    """The die-split tile order alone, for profiling it: the 8192^3 bf16
    2-CTA GEMM (fp32 C) launched once to warm up and twice in the plain
    order, then twice with the measured die map installed; the outputs
    compared bit for bit."""
    import cuda_micro_bench_b200 as cmbpkg
    from cuda_micro_bench_b200 import check

    M = N = K = 8192
    A = torch.empty(M * K, dtype=torch.int16, device="cuda")
    B = torch.empty(N * K, dtype=torch.int16, device="cuda")
    check("cmb_fill_normal_bf16", ctypes.c_void_p(A.data_ptr()), M * K, ctypes.c_uint64(SEED + 1),
          ctypes.c_float(K ** -0.5), sh)
    check("cmb_fill_normal_bf16", ctypes.c_void_p(B.data_ptr()), N * K, ctypes.c_uint64(SEED + 2),
          ctypes.c_float(K ** -0.5), sh)
    C = torch.empty(M * N, dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    labels, out = install_die_map(sh)
    fn = lambda: check("cmb_gemm_bf16", ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                       ctypes.c_void_p(C.data_ptr()), M, N, K, 2,
                       ctypes.c_void_p(status.data_ptr()), sh)
    cmbpkg.set_sm_die_map(None)
    fn()  # warm-up: the first launch of the kernel in this process
    ms = _time_launches(torch, stream, fn, 2)
    plain = C.clone()
    cmbpkg.set_sm_die_map(labels)
    ms += _time_launches(torch, stream, fn, 2)
    out["launch_ms_plain_plain_split_split"] = [round(x, 4) for x in ms]
    out["bit_equal_to_plain_order"] = bool(torch.equal(C, plain))
    out["status"] = int(status.item())
    cmbpkg.set_sm_die_map(None)
    return out


def probe_copy_forms(torch, stream, sh) -> dict:
    """The 4 GiB device copy by every engine this library drives, for
    placing the copy stream against the device's own copy ceiling: the
    load/store-unit stream (cmb_stream_copy), the peer-store kernel on one
    local job, bulk copies through shared memory (the P2P bulk kernel on one
    local job, several chunk / ring / CTA shapes) and the copy engines
    (cudaMemcpyAsync device to device through torch).  GB/s = 2 x 4 GiB /
    median of 12 launches after 3 warm-up launches; every output compared
    with the source bit for bit."""
    from cuda_micro_bench_b200 import check

    n = 1 << 30
    nbytes = 4 * n
    src = torch.empty(n, dtype=torch.float32, device="cuda")
    dst = torch.empty(n, dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    check("cmb_fill_uniform_f32", ctypes.c_void_p(src.data_ptr()), n, ctypes.c_uint64(SEED), sh)
    D = (ctypes.c_void_p * 1)(dst.data_ptr())
    S = (ctypes.c_void_p * 1)(src.data_ptr())
    NB = (ctypes.c_size_t * 1)(nbytes)
    forms = {
        "stream_copy": lambda: check("cmb_stream_copy", ctypes.c_void_p(dst.data_ptr()),
                                     ctypes.c_void_p(src.data_ptr()), nbytes, sh),
        "peer_store_kernel_local": lambda: check("cmb_p2p_scatter_store", D, S, NB, 1, 0, sh),
        "copy_engine_d2d": lambda: dst.copy_(src),
    }
    for chunk, stages, ctas in ((16384, 4, 148), (16384, 8, 148), (32768, 4, 148),
                                (8192, 4, 444)):
        forms[f"bulk_{chunk // 1024}k_{stages}stages_{ctas}ctas"] = (
            lambda chunk=chunk, stages=stages, ctas=ctas: check(
                "cmb_p2p_scatter_bulk_tuned", D, S, NB, 1, ctas, chunk, stages,
                ctypes.c_void_p(status.data_ptr()), sh))
    out = {}
    for name, fn in forms.items():
        dst.zero_()
        ms = _median_ms(torch, stream, fn, reps=12, warm=3)
        out[name] = {"GB/s": round(2 * nbytes / (ms * 1e-3) / 1e9, 1),
                     "bit_exact": bool(torch.equal(dst, src)), "status": int(status.item())}
    del src, dst
    return out


def run_probe_only(args) -> int:
    """Runs only the named probes (for profiling) and prints their results."""
    import torch

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    peaks = measured_peaks()
    out = {}
    for name in args.probe:
        if name == "stream":
            out.update(probe_stream_1gib(torch, stream, sh, peaks))
        elif name == "chase":
            out["chase_512mib"] = probe_chase(torch, stream, sh, 1 << (22 if args.quick_chase else 24))
        elif name == "tma":
            out["tma_16384"] = probe_tma(torch, stream, sh, peaks)
        elif name == "gemm":
            out["gemm"] = probe_gemm(torch, stream, sh, peaks)
        elif name == "cublas":
            out["cublas_8192"] = probe_cublas(torch, stream, sh)
        elif name == "gemm256":
            out["gemm_256x256"] = probe_cublas(torch, stream, sh, ours_tile256=True)
        elif name == "gemm_die":
            out["gemm_die"] = probe_gemm_die(torch, stream, sh)
        elif name == "copy_forms":
            out["copy_forms_4gib"] = probe_copy_forms(torch, stream, sh)
        torch.cuda.empty_cache()
    print(json.dumps({"probes": out}), flush=True)
    return 0


def cpu_probe_baselines() -> dict:
    """The host reference of the other probes, timed on this box's cores on
    bounded samples (the oracle: threaded fp64 sum, the serial chase walk,
    threaded blocked fp32 GEMM rows)."""
    import numpy as np

    import oracle

    orc = oracle.load()
    threads = orc.orc_hw_threads()
    out = {"cores": threads}
    n = 1 << 28
    x = np.empty(n, np.float32)
    orc.orc_fill_uniform_f32(oracle.ptr(x), n, SEED)
    t0 = time.perf_counter()
    orc.orc_sum_f64(oracle.ptr(x), n, threads)
    dt = time.perf_counter() - t0
    out["sum_1gib"] = {"GB/s": round(4.0 * n / dt / 1e9, 2), "threads": threads,
                       "sample": "fp64 sum of fp32[2^28]"}
    del x
    links = np.empty((512 << 20) // 4, np.uint32)
    orc.orc_chase_build(oracle.ptr(links), links.nbytes, 0xC0DA)
    hops = 1 << 22
    t0 = time.perf_counter()
    orc.orc_chase_walk(oracle.ptr(links), hops, 0)
    dt = time.perf_counter() - t0
    out["chase_512mib"] = {"ns_per_hop": round(dt * 1e9 / hops, 2), "threads": 1,
                           "sample": "serial walk, 2^22 hops over 512 MiB"}
    del links
    K, N, rows = 8192, 8192, 64 * threads
    # N(0, 1/K) operands, as the GPU probe fills them, truncated to bf16
    bf16 = lambda x: (x.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    a = bf16(np.random.default_rng(0).standard_normal(rows * K, np.float32) * K ** -0.5)
    b = bf16(np.random.default_rng(1).standard_normal(N * K, np.float32) * K ** -0.5)
    c = np.empty(rows * N, np.float32)
    t0 = time.perf_counter()
    orc.orc_gemm_bf16_rows_f32(oracle.ptr(a), oracle.ptr(b), oracle.ptr(c), N, K, 0, rows, threads)
    dt = time.perf_counter() - t0
    out["gemm_bf16"] = {"TFLOP/s": round(2.0 * rows * N * K / dt / 1e12, 5), "threads": threads,
                        "sample": f"{rows} rows of an 8192^3 bf16 GEMM (blocked fp32)"}
    return out


def run_probes(args, ranks, peaks) -> dict:
    import torch

    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    out = {}
    if ranks.world > 1:
        out["p2p_256mib"] = probe_p2p(args, ranks)
    if ranks.world == 1:
        out.update(probe_stream_1gib(torch, stream, sh, peaks))
        out["chase_512mib"] = probe_chase(torch, stream, sh, 1 << (22 if args.quick_chase else 24))
        torch.cuda.empty_cache()
        out["tma_16384"] = probe_tma(torch, stream, sh, peaks)
        torch.cuda.empty_cache()
        out["gemm"] = probe_gemm(torch, stream, sh, peaks)
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------- reference arm


def run_reference(args) -> int:
    """The reference arm: the CPU implementation of the same copy (the
    oracle's threaded memcpy) on the host cores, rank 0 only; one step = one
    memcpy of a bounded sample (1 GiB, or 256 MiB when K > 64) so the K
    steps finish within a minute or two."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sample = (1 << 30) if args.steps <= 64 else (256 << 20)
    warm = max(1, min(args.warmup, 3))
    base = cpu_memcpy_baseline(sample, args.steps, warm)
    result = {
        "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * base["seconds"] / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded bytes, SplitMix64)",
        "config": {"workload": "stream_copy on host cores: memcpy sample of the per-GPU copy",
                   "parallelism": "host threads", "impl": "reference"},
        "impl": "reference", "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=3, help="0 skips the e2e leg")
    ap.add_argument("--gib", type=float, default=4.0, help="copy size per GPU in GiB (default 4)")
    ap.add_argument("--no-probes", action="store_true", help="headline only")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick-chase", action="store_true",
                    help="2^22 chase hops instead of the configuration's 2^24")
    ap.add_argument("--probe", action="append",
                    choices=["stream", "chase", "tma", "gemm", "cublas", "gemm256", "gemm_die",
                             "copy_forms"],
                    help="run only this probe (repeatable); no headline line")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        # at least 3 untimed warm-up steps always run; the line reports the count used
        log(f"--warmup {args.warmup} raised to 3")
        args.warmup = 3
    if args.steps < 1:
        ap.error("--steps must be >= 1")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus != world:
        ap.error(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if args.impl == "reference":
        return run_reference(args)
    if args.probe:
        return run_probe_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
