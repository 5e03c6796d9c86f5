#!/usr/bin/env python
"""Benchmark of librocketnpu's matmul hot path on B200.

Headline workload: the 12B-class prefill GEMM set with
int8 per-output-channel weights, M = 4096 tokens:
    QKV     K=3840  N=5888
    O-proj  K=3840  N=3840
    gate+up K=3840  N=30720
    down    K=15360 N=3840
1755.57 GOP per set.  One step = the four GEMMs through the reference API
(rocket_matmul_int8_prepacked on a resident rocket_i8_weights), raw int32
outputs, bit-exact to the reference's host int64 sum.

Multi-GPU (torchrun): every weight is N-sharded across the ranks (the
reference's worker N-split), each rank holds its column slice and the full A,
and computes its slice with no collective; total work is fixed, so scaling is
"strong".  The NCCL all-gather of the outputs (only needed when a caller wants
the full output on one rank) is timed separately and reported, not included.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

M_TOK = 4096
GEMMS = [("qkv", 3840, 5888), ("o_proj", 3840, 3840), ("gate_up", 3840, 30720), ("down", 15360, 3840)]
SET_OPS = sum(2.0 * M_TOK * k * n for _, k, n in GEMMS)          # 1.75557e12
METRIC = "int8 TOPS at 12B-prefill GEMM set (config 5), % of B200 dense int8 peak"
WORKLOAD = "12B prefill int8 GEMM set M=4096: QKV 3840x5888, O 3840x3840, gate+up 3840x30720, down 15360x3840"
NOMINAL_INT8_TOPS = 4500.0
NOMINAL_F16_TFLOPS = 2250.0


def load_pkg():
    """Import rocket-userspace_b200/ (its directory name is not an identifier)."""
    import importlib.util
    if "rocket_userspace_b200" in sys.modules:
        return sys.modules["rocket_userspace_b200"]
    pkg = os.path.join(REPO, "rocket-userspace_b200")
    spec = importlib.util.spec_from_file_location("rocket_userspace_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["rocket_userspace_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def shard(n, world, rank, atom=32):
    """Column slice of `rank` (rocket-userspace_b200/shard.py, the reference's worker split)."""
    return load_pkg().shard.shard(n, world, rank, atom)


class Clocks:
    """SM clock, power and clock-event reasons sampled through NVML every ~2 ms
    on a background thread (reading only; nothing is set), so that even a
    timed region of a few milliseconds holds samples.  Only samples taken
    between mark("t_start") and mark("t_end") are kept; when the region is
    shorter than one sampling interval the samples on either side of it are
    reported instead (and `bracketing` says so)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, idx):
        self.idx = idx
        self.samples = []
        self.stop_flag = False
        self.thread = None
        self.sm_max = None
        self.t_start, self.t_end = 0.0, 1e30

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:   # noqa: BLE001 -- no NVML: report that, do not fail the bench
            self.thread = None
            return

        def run():
            while not self.stop_flag:
                try:
                    t = time.time()
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                    self.samples.append((t, sm, pw, rs))
                except Exception:   # noqa: BLE001
                    pass
                time.sleep(0.002)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML unavailable"],
                    "samples_in_timed_region": 0}
        time.sleep(0.01)
        self.stop_flag = True
        self.thread.join(timeout=5)
        inside = [x for x in self.samples if self.t_start <= x[0] <= self.t_end]
        bracketing = False
        if not inside:
            before = [x for x in self.samples if x[0] < self.t_start][-1:]
            after = [x for x in self.samples if x[0] > self.t_end][:1]
            inside, bracketing = before + after, True
        reasons = sorted({nm for _, _, _, rs in inside for nm, bit in self.REASONS.items() if rs & bit})
        sm = [x[1] for x in inside]
        pw = [x[2] for x in inside]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.sm_max,
                "reasons": reasons, "samples_in_timed_region": 0 if bracketing else len(inside),
                "bracketing": bracketing, "sampler": "NVML, 2 ms",
                "timed_region_s": self.t_end - self.t_start,
                "power_w_median": statistics.median(pw) if pw else None}


# ---------------------------------------------------------------- CPU baseline
def cpu_baseline(seconds=10.0):
    """The reference's host matmul (int64-accumulate loop, restated in the
    oracle and pinned by the reference's gates) on this host's cores, over a
    bounded sample of gate+up rows; TOPS = ops done / time.  Timed twice: on
    one thread (the loop as the reference's gates run it) and on every core
    (rows split across threads)."""
    import oracle
    cores = os.cpu_count() or 1
    K, N = 3840, 30720
    A = oracle.uniform_i8(1, -127, 127, (M_TOK, K))
    B = oracle.uniform_i8(2, -127, 127, (N, K))

    def timed(nthreads, budget, chunk):
        rows, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget and rows + chunk <= M_TOK:
            oracle.matmul_int8(A, B, rows=(rows, rows + chunk), nthreads=nthreads)
            rows += chunk
        return rows, time.perf_counter() - t0

    r1, t1 = timed(1, seconds / 3, 1)
    rn, tn = timed(cores, 2 * seconds / 3, max(cores, 8))
    single = 2.0 * r1 * K * N / t1 / 1e12
    tops = 2.0 * rn * K * N / tn / 1e12
    return {"value": tops, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": f"{rn} rows of the gate+up GEMM (K=3840, N=30720) in {tn:.1f}s on {cores} threads, "
                      "int64-accumulate host loop of tests/matmul_int8_tiled_rocket.c:77-83 "
                      "(oracle/oracle.c orc_matmul_int8, -O2), rows split across cores",
            "rows": rn, "seconds": tn,
            "single_thread": {"value": single, "unit": "TOPS", "cores": 1, "rows": r1, "seconds": t1,
                              "sample": f"{r1} rows of the gate+up GEMM on one thread in {t1:.1f}s"}}


def run_reference(args):
    """The reference arm: the reference's own host matmul loop on this box's
    host cores.  One bounded sample is measured (not args.steps full steps:
    a full step is ~1.76 TOP, minutes of CPU time); the line says so."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    base = cpu_baseline(seconds=20.0)
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "TOPS",
            "n_gpus": args.gpus, "steps": 1, "steps_requested": args.steps, "warmup": 0,
            "ms_per_step": SET_OPS / (base["value"] * 1e12) * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sampled": True},
            "extrapolated": True,
            "measured": {"rows_computed": base["rows"], "of_rows_per_step": M_TOK,
                         "gemm_sampled": "gate+up (K=3840, N=30720)", "seconds": base["seconds"]},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference's own host matmul (its gates' int64 loop) on the host cores, over a sample of "
                    "rows; ms_per_step is extrapolated from that sample to the whole GEMM set. The reference "
                    "library's matmul needs an RK3588 NPU, which this box does not have"}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm
def main_ours(args):
    import ctypes
    import torch
    rank, world, local = dist_env()
    os.environ["ROCKET_DEV"] = str(local)
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rkb = load_pkg()
    L = rkb.lib
    peaks, peak_src = load_peaks()

    # one resident context per GEMM of the set (each owns a handle and a CUDA
    # stream), so the four independent GEMMs of a step can run concurrently and
    # fill each other's partial last waves; --streams 1 puts all on one context
    nctx = len(GEMMS) if args.streams > 1 else 1
    ctxs = [L.rocket_i8_ctx_create(1) for _ in range(nctx)]
    assert all(ctxs), "rocket_i8_ctx_create failed"
    ctx = ctxs[0]
    dev_t = torch.device("cuda", local)
    lib_streams = [torch.cuda.ExternalStream(L.rocket_b200_stream(L.rocket_b200_ctx_fd(c, 0)), device=dev_t)
                   for c in ctxs]
    lib_stream = lib_streams[0]

    g = torch.Generator(device="cuda")
    g.manual_seed(1234 + rank)
    A1 = torch.randint(-127, 128, (M_TOK, 3840), dtype=torch.int8, device="cuda", generator=g)
    A2 = torch.randint(-127, 128, (M_TOK, 15360), dtype=torch.int8, device="cuda", generator=g)
    layers = []
    my_ops = 0.0
    for gi, (name, K, N) in enumerate(GEMMS):
        if args.layers and name not in args.layers.split(","):
            continue
        n0, ns = shard(N, world, rank)
        cx = ctxs[gi % nctx]
        W = torch.randint(-127, 128, (ns, K), dtype=torch.int8, device="cuda", generator=g)
        w = L.rocket_i8_weights_pack(cx, M_TOK, K, ns, W.data_ptr())
        assert w, f"pack {name}"
        del W
        C = torch.empty((M_TOK, ns), dtype=torch.int32, device="cuda")
        A = A1 if K == 3840 else A2
        layers.append((name, K, ns, w, A, C, cx))
        my_ops += 2.0 * M_TOK * K * ns
    torch.cuda.synchronize()

    def step(As=None, Cs=None):
        for i, (name, K, ns, w, A, C, cx) in enumerate(layers):
            a = A if As is None else As[i]
            c = C if Cs is None else Cs[i]
            rc = L.rocket_matmul_int8_prepacked(cx, M_TOK, K, ns, a.data_ptr(), c.data_ptr(), w)
            if rc != 0:
                raise RuntimeError(f"{name}: rc={rc}")

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timed region
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.05)
    # the timed region runs without the per-kernel profiler: its CUDA events
    # between kernels cost device time; kernel durations come from a separate
    # profiled pass below
    L.rocket_b200_profile_enable(0)
    L.rocket_submit_counters_reset()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # device-resident operands: enqueue every call of the timed region without
    # waiting (rocket_b200_set_async), then one rocket_b200_ctx_sync collects
    # the status of all of them
    L.rocket_b200_set_async(1)
    main = torch.cuda.current_stream()
    clocks.mark("t_start")
    e0.record(main)
    for st in lib_streams:
        st.wait_event(e0)
    for _ in range(args.steps):
        step()
    for st in lib_streams:
        ev = torch.cuda.Event()
        ev.record(st)
        main.wait_event(ev)
    e1.record(main)
    rc_sync = 0
    for c in ctxs:
        rc_sync = rc_sync or L.rocket_b200_ctx_sync(c)
    clocks.mark("t_end")
    L.rocket_b200_set_async(0)
    assert rc_sync == 0, f"ctx_sync {rc_sync}"
    torch.cuda.synchronize()
    barrier()
    launches = int(L.rocket_submit_task_count())
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    # profiled pass: per-kernel CUDA events on the library streams; calls
    # are synchronous here, so kernels run one at a time and each launch's
    # duration is its own
    prof_steps = max(1, min(args.steps, 50))
    L.rocket_b200_profile_reset()
    L.rocket_b200_profile_enable(1)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    p0.record(main)
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    p1.record(main)
    torch.cuda.synchronize()
    L.rocket_b200_profile_enable(0)
    prof_ms = p0.elapsed_time(p1)
    ms_max = max_over_ranks(ms)
    step_ops = SET_OPS if not args.layers else sum(
        2.0 * M_TOK * k * n for nm, k, n in GEMMS if nm in args.layers.split(","))
    value = step_ops * args.steps / (ms_max / 1e3) / 1e12
    prof = rkb.profile_snapshot()
    n_i8, ms_i8 = prof.get("gemm_i8_tcgen05", (0, 0.0))

    # roofline of the dominant kernel (the int8 GEMM), per launch
    ops_per_launch = my_ops / len(layers)
    # prof_ms spans host gaps between the synchronous calls: the kernel share
    # below is a lower bound
    avg_launch_ms = ms_i8 / max(n_i8, 1)
    achieved = ops_per_launch / (avg_launch_ms / 1e3) / 1e12
    derived_peak = 2.0 * peaks.get("bf16_tflops", 1590.0)
    sustained_peak = 2.0 * peaks.get("bf16_tflops_sustained", 1400.0)
    # burst vs sustained from this run's own clock record: a timed region whose
    # samples show the power cap ran at capped clocks (the sustained rate was
    # measured the same way); one without runs at the burst rate
    capped = "sw_power_cap" in clk.get("reasons", [])
    long_capped = capped
    peak = sustained_peak if long_capped else derived_peak
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS",
                "frac": achieved / peak, "traffic": None,
                "peak_source": (f"2 x {peak_src} bf16 {'sustained' if long_capped else 'burst'} "
                                f"({peaks.get('bf16_tflops_sustained' if long_capped else 'bf16_tflops')} TF/s): "
                                f"the timed region lasted {ms / 1e3:.3f} s with power-cap samples "
                                f"{'present' if capped else 'absent'}. B200 dense int8 rate is twice its "
                                "bf16 rate; no int8 figure in MEASURED_PEAKS.json"),
                "frac_of_2x_sustained_bf16": achieved / sustained_peak,
                "frac_of_2x_burst_bf16": achieved / derived_peak,
                "frac_of_nominal_4500": achieved / NOMINAL_INT8_TOPS,
                "kernel": "gemm_i8_tcgen05", "launches": n_i8,
                "avg_launch_us": avg_launch_ms * 1e3,
                "profiled_pass": f"{prof_steps} steps with per-kernel events, apart from the timed region",
                "kernel_share_of_step": ms_i8 / prof_ms if prof_ms > 0 else None}
    traffic_file = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(traffic_file):
        roofline["traffic"] = json.load(open(traffic_file)).get("gemm_i8_config5_avg_launch_bytes")

    # ---- all-gather of the sharded outputs (reported, not in value)
    gather = None
    if world > 1:
        import torch.distributed as dist
        bufs = []
        for name, K, ns, w, A, C, cx in layers:
            n0, nmax = shard(dict((a, b) for a, _, b in GEMMS)[name], world, 0)
            src = torch.zeros((M_TOK, nmax), dtype=torch.int32, device="cuda")
            src[:, :ns] = C
            bufs.append((src, torch.empty((world, M_TOK, nmax), dtype=torch.int32, device="cuda")))
        for src, dst in bufs:
            dist.all_gather_into_tensor(dst, src)
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(3):
            for src, dst in bufs:
                dist.all_gather_into_tensor(dst, src)
        g1.record()
        torch.cuda.synchronize()
        gms = max_over_ranks(g0.elapsed_time(g1) / 3)
        gather = {"allgather_ms_per_step": gms, "collective": "nccl all_gather_into_tensor",
                  "value_with_gather": SET_OPS / ((ms_max / args.steps + gms) / 1e3) / 1e12}

    # ---- end to end through the API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        hA = [torch.empty_like(ly[4], device="cpu").pin_memory() for ly in layers]
        for h, ly in zip(hA, layers):
            h.copy_(ly[4].cpu())
        hC = [torch.empty(ly[5].shape, dtype=torch.int32).pin_memory() for ly in layers]
        e2e_steps = max(1, min(args.steps, 20))
        step(hA, hC)
        torch.cuda.synchronize()
        barrier()
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(main)
        for _ in range(e2e_steps):
            step(hA, hC)
        torch.cuda.synchronize()
        x1.record(main)
        torch.cuda.synchronize()
        ems = max_over_ranks(x0.elapsed_time(x1))
        ok = all(torch.equal(hC[i], layers[i][5].cpu()) for i in range(len(layers)))
        e2e = {"value": step_ops * e2e_steps / (ems / 1e3) / 1e12, "unit": "TOPS",
               "h2d_bytes_per_step": int(sum(h.numel() for h in hA)) * world,
               "d2h_bytes_per_step": int(sum(h.numel() * 4 for h in hC)) * world,
               "steps": e2e_steps, "host_result_matches_device": ok,
               "path": "rocket_matmul_int8_prepacked with pinned host A and C (H2D + D2H inside each call)"}

    # ---- other configs (rank 0, N=1 only)
    others = None
    if world == 1 and not args.no_extra:
        others = other_configs(rkb, torch, peaks, derived_peak,
                               tuple(args.side.split(",")) if args.side else ("c1", "c2", "c3", "c4", "ops", "fa"))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(seconds=10.0)

    for name, K, ns, w, A, C, cx in layers:
        L.rocket_i8_weights_free(cx, w)
    for c in ctxs:
        L.rocket_i8_ctx_free(c)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8 (s8 x s8 -> s32, exact)",
                "data": "synthetic: int8 uniform [-127,127], seeded",
                "config": {"workload": WORKLOAD, "M": M_TOK, "ops_per_step": SET_OPS,
                           "parallelism": f"N-shard x{world}", "l2": "working set per step ~1 GB > 126 MB L2 (no flush needed)",
                           "api": "rocket_matmul_int8_prepacked on device-resident operands, enqueued with rocket_b200_set_async(1) and one rocket_b200_ctx_sync per context per timed region",
                           "streams": nctx, "concurrency": ("each GEMM of the set on its own resident context and CUDA stream; the four independent GEMMs of consecutive steps overlap"
                                                            if nctx > 1 else "one context, one stream: GEMMs run one after another")},
                "frac_of_sustained_int8_peak": value / sustained_peak, "frac_of_burst_int8_peak": value / derived_peak,
                "roofline": roofline, "clocks": clk, "gpu_launches": launches,
                "e2e": e2e, "cpu_baseline": cpu, "gather": gather, "other_configs": others}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def other_configs(rkb, torch, peaks, derived_i8_peak, which=("c1", "c2", "c3", "c4", "ops", "fa")):
    """fp16 (config 2), W4A8 group-wise (config 3) and int8 latency (config 1)."""
    L = rkb.lib
    out = {}
    dev = rkb.Device()
    stream = torch.cuda.ExternalStream(L.rocket_b200_stream(dev.fd))

    def timed(fn, n):
        """Device time per call: device-resident operands enqueued back to back
        (rocket_b200_set_async), CUDA events on the handle's stream."""
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        L.rocket_b200_set_async(1)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        rc = L.rocket_b200_sync(dev.fd)
        L.rocket_b200_set_async(0)
        assert rc == 0, rc
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    def kernel_ms(fn, n, family):
        """Mean device duration of the library's kernels of `family` (CUDA events
        around each launch on its own stream, rocket_b200_profile_*)."""
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        L.rocket_b200_profile_reset()
        L.rocket_b200_profile_enable(1)
        L.rocket_b200_set_async(1)   # back to back: events bracket device work only
        for _ in range(n):
            fn()
        rc = L.rocket_b200_sync(dev.fd)
        L.rocket_b200_set_async(0)
        L.rocket_b200_profile_enable(0)
        assert rc == 0, rc
        cnt, tot = rkb.profile_snapshot().get(family, (0, 0.0))
        return tot / max(cnt, 1)

    # config 2: fp16 512x4096x4096
    if "c2" in which:
        M, K, N = 512, 4096, 4096
        A = (torch.randn((M, K), device="cuda") / K ** 0.5).half()
        B = (torch.randn((N, K), device="cuda") / K ** 0.5).half()
        C = torch.empty((M, N), dtype=torch.float16, device="cuda")
        ms = timed(lambda: dev.matmul_fp16(M, K, N, A, B, C), 200)
        ref = torch.matmul(A, B.t())
        for _ in range(3):
            torch.matmul(A, B.t())
        ta, tb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ta.record()
        for _ in range(200):
            torch.matmul(A, B.t())
        tb.record()
        torch.cuda.synchronize()
        t = ta.elapsed_time(tb) / 200
        kms = kernel_ms(lambda: dev.matmul_fp16(M, K, N, A, B, C), 50, "gemm_f16_tcgen05")
        out["config2_fp16"] = {"tflops": 2 * M * N * K / ms / 1e9, "ms": ms,
                               "kernel_tflops": 2 * M * N * K / kms / 1e9, "kernel_ms": kms,
                               "frac_of_measured_bf16": 2 * M * N * K / ms / 1e9 / peaks["bf16_tflops"],
                               "torch_cublas_tflops": 2 * M * N * K / t / 1e9,
                               "rel_fro_vs_cublas": float((C.float() - ref.float()).norm() / ref.float().norm())}
        # large fp16 for the kernel's steady-state rate
        M2 = 4096
        A2 = torch.randn((M2, K), device="cuda").half()
        C2 = torch.empty((M2, N), dtype=torch.float16, device="cuda")
        ms2 = timed(lambda: dev.matmul_fp16(M2, K, N, A2, B, C2), 30)
        out["fp16_4096x4096x4096"] = {"tflops": 2 * M2 * N * K / ms2 / 1e9,
                                      "frac_of_measured_bf16": 2 * M2 * N * K / ms2 / 1e9 / peaks["bf16_tflops"]}
        del A2, C2

    # config 3: W4A8 group-wise resident 2048x3840x15360, group 32
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if "c3" in which:
        M, K, N, gsz = 2048, 3840, 15360, 32
        nG = K // gsz
        ctx = L.rocket_i4_ctx_create(1)
        Wt = torch.randint(-8, 8, (N, K), dtype=torch.int8, device="cuda")
        w = L.rocket_i4_weights_pack_gw(ctx, M, K, N, Wt.data_ptr(), gsz)
        Aq = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
        asc = (torch.rand((M, 1), device="cuda") * 0.04 + 0.01).expand(M, nG).contiguous()
        bsc = torch.rand((N, nG), device="cuda") * 0.015 + 0.005
        Cf = torch.empty((M, N), dtype=torch.float32, device="cuda")
        fd3 = L.rocket_b200_ctx_fd(ctx, 0)
        s3 = torch.cuda.ExternalStream(L.rocket_b200_stream(fd3))
        run3 = lambda: L.rocket_matmul_int4_prepacked_gw(ctx, M, K, N, Aq.data_ptr(), asc.data_ptr(),
                                                         bsc.data_ptr(), Cf.data_ptr(), w)
        res3 = {}
        for mode, mname, fam in ((0, "precise", "wgemm_gw_i8_tcgen05"), (1, "fast", "wgemm_w4_f16_tcgen05")):
            L.rocket_b200_gw_mode(mode)
            for _ in range(3):
                run3()
            torch.cuda.synchronize()
            # device time per call: group-wise calls wait for their stream, so
            # each call's host round trip is inside this figure
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s3)
            for _ in range(20):
                run3()
            b.record(s3)
            torch.cuda.synchronize()
            ms3 = a.elapsed_time(b) / 20
            L.rocket_b200_profile_reset()
            L.rocket_b200_profile_enable(1)
            for _ in range(20):
                run3()
            torch.cuda.synchronize()
            L.rocket_b200_profile_enable(0)
            prof = rkb.profile_snapshot()
            nk, kms = prof.get(fam, (1, 0.0))
            res3[mname] = {"tops_call": 2 * M * N * K / ms3 / 1e9, "ms_call": ms3,
                           "kernel_tops": 2 * M * N * K / (kms / max(nk, 1)) / 1e9,
                           "kernel_frac_of_measured_f16": 2 * M * N * K / (kms / max(nk, 1)) / 1e9 / peaks["bf16_tflops"],
                           "per_call_kernels": {k: v for k, v in prof.items() if v[0]}}
        L.rocket_b200_gw_mode(0)
        res3["note"] = ("precise (default): exact int32 partial per 32-wide group from the int8 MMA on the unscaled "
                        "operands, scaled and summed in fp32 (the reference's definition, its gates' 1e-5 rms bound); "
                        "fast: w*scale rounded to fp16 in-register before the MMA (north-star 1e-2 bound). "
                        "Fractions are of the fp16 dense rate; the precise kernel runs int8 MMAs, whose peak is twice that")
        out["config3_w4a8_gw"] = res3
        L.rocket_i4_weights_free(ctx, w)
        L.rocket_i4_ctx_free(ctx)

    # config 4: encoder block fp16, d=512, 8 heads, T=1500, batch 4 (batched extension)
    if "c4" in which:
        nb, T, d, nh, dff = 4, 1500, 512, 8, 2048
        BT = nb * T
        gq = torch.Generator(device="cuda")
        gq.manual_seed(4)
        pw = {}
        for k, shp in [("Wq", (d, d)), ("Wk", (d, d)), ("Wv", (d, d)), ("Wo", (d, d)), ("W1", (dff, d)), ("W2", (d, dff))]:
            pw[k] = (torch.randn(shp, device="cuda", generator=gq) * 0.02).half()
        for k, n in [("bq", d), ("bk", d), ("bv", d), ("bo", d), ("b1", dff), ("b2", d)]:
            pw[k] = (torch.randn(n, device="cuda", generator=gq) * 0.02).half()
        for k in ("ln1_g", "ln2_g"):
            pw[k] = torch.ones(d, device="cuda", dtype=torch.float16)
        for k in ("ln1_b", "ln2_b"):
            pw[k] = torch.zeros(d, device="cuda", dtype=torch.float16)
        xe = torch.randn((BT, d), device="cuda", generator=gq).half()
        ye = torch.empty_like(xe)
        run4 = lambda: L.rocket_b200_encoder_block_batched_fp16(dev.fd, nb, T, d, nh, dff, xe.data_ptr(),
                                                                *[pw[k].data_ptr() for k in rkb.ENCODER_KEYS],
                                                                1e-5, ye.data_ptr())
        flops4 = (2.0 * BT * d * 3 * d + 2.0 * BT * d * d + 2 * 2.0 * nb * nh * T * T * (d // nh)
                  + 2 * 2.0 * BT * d * dff)
        for _ in range(3):
            assert run4() == 0
        torch.cuda.synchronize()
        # device time per block: device-resident operands, calls enqueued back to
        # back (rocket_b200_set_async), no profiler events
        L.rocket_b200_set_async(1)
        a.record(stream)
        for _ in range(10):
            run4()
        b.record(stream)
        assert L.rocket_b200_sync(dev.fd) == 0
        L.rocket_b200_set_async(0)
        torch.cuda.synchronize()
        ms4 = a.elapsed_time(b) / 10
        # LayerNorm alone, HBM roofline: [100000, 512] fp16 (205 MB moved per call > 126 MB L2)
        LN_ROWS = 100000
        xl = torch.randn((LN_ROWS, d), device="cuda", generator=gq).half()
        yl = torch.empty_like(xl)
        runln = lambda: L.rocket_layernorm_fp16(dev.fd, LN_ROWS, d, xl.data_ptr(), pw["ln1_g"].data_ptr(),
                                                pw["ln1_b"].data_ptr(), 1e-5, yl.data_ptr())
        for _ in range(3):
            assert runln() == 0
        L.rocket_b200_set_async(1)
        a.record(stream)
        for _ in range(200):
            runln()
        b.record(stream)
        assert L.rocket_b200_sync(dev.fd) == 0
        L.rocket_b200_set_async(0)
        torch.cuda.synchronize()
        ms_ln_call = a.elapsed_time(b) / 200
        # kernel durations: a separate profiled pass
        L.rocket_b200_profile_reset()
        L.rocket_b200_profile_enable(1)
        for _ in range(10):
            run4()
        torch.cuda.synchronize()
        L.rocket_b200_profile_enable(0)
        prof = rkb.profile_snapshot()
        n_ln, ms_ln = prof.get("norm", (1, 0.0))
        ln_bytes = 2.0 * LN_ROWS * d * 2 + 2 * d * 2
        n_at, ms_at = prof.get("attention", (1, 0.0))
        at_flops = 2 * 2.0 * nb * nh * T * T * (d // nh)
        out["config4_encoder_block"] = {
            "tflops": flops4 / ms4 / 1e9, "ms": ms4, "gflop": flops4 / 1e9,
            "layernorm_gbs": ln_bytes / (ms_ln_call / 1e3) / 1e9,
            "layernorm_frac_of_measured_hbm": ln_bytes / (ms_ln_call / 1e3) / 1e9 / peaks["hbm_gbs"],
            "layernorm_us": ms_ln_call * 1e3,
            "layernorm_note": "rocket_layernorm_fp16 on a [100000, 512] fp16 tensor (read + write 205 MB > L2), 200 calls enqueued back to back, device pointers, no profiler",
            "attention_tflops": at_flops / (ms_at / max(n_at, 1) / 1e3) / 1e12,
            "per_kernel_ms": {k: v[1] / 10 for k, v in prof.items() if v[0]},
            "note": "batched over 4 sequences via rocket_b200_encoder_block_batched_fp16"}

    # HBM-bound encoder ops standalone, at sizes above L2 (126 MB): achieved
    # GB/s = bytes read + written per call / device time per call
    if "ops" in which:
        res = {}
        go = torch.Generator(device="cuda")
        go.manual_seed(5)
        SM_R, SM_N = 48000, 1500            # softmax rows of config-4 attention scores (32 heads x 1500)
        xs = torch.randn((SM_R, SM_N), device="cuda", generator=go).half()
        ys = torch.empty_like(xs)
        ms = timed(lambda: L.rocket_softmax_fp16(dev.fd, SM_R, SM_N, xs.data_ptr(), ys.data_ptr()), 50)
        res["softmax_48000x1500"] = {"us": ms * 1e3, "gbs": 2 * xs.numel() * 2 / (ms / 1e3) / 1e9}
        del xs, ys
        NE = 1 << 26
        xa = torch.randn(NE, device="cuda", generator=go).half()
        xb = torch.randn(NE, device="cuda", generator=go).half()
        yo = torch.empty_like(xa)
        ms = timed(lambda: L.rocket_activation_fp16(dev.fd, 5, xa.data_ptr(), yo.data_ptr(), NE), 50)
        res["gelu_64Mi"] = {"us": ms * 1e3, "gbs": 2 * NE * 2 / (ms / 1e3) / 1e9}
        ms = timed(lambda: L.rocket_ew_add_fp16(dev.fd, xa.data_ptr(), xb.data_ptr(), yo.data_ptr(), NE), 50)
        res["ew_add_64Mi"] = {"us": ms * 1e3, "gbs": 3 * NE * 2 / (ms / 1e3) / 1e9}
        del xa, xb, yo
        RN, RH = 100000, 512
        xr = torch.randn((RN, RH), device="cuda", generator=go).half()
        gr = torch.ones(RH, device="cuda", dtype=torch.float16)
        yr = torch.empty_like(xr)
        ms = timed(lambda: L.rocket_rmsnorm_fp16(dev.fd, RN, RH, xr.data_ptr(), gr.data_ptr(), 1e-6,
                                                 yr.data_ptr()), 50)
        res["rmsnorm_100000x512"] = {"us": ms * 1e3, "gbs": 2 * xr.numel() * 2 / (ms / 1e3) / 1e9}
        for v in res.values():
            v["frac_of_measured_hbm"] = v["gbs"] / peaks["hbm_gbs"]
        out["hbm_ops"] = res

    # masked grouped-query flash attention (rocket_flash_attn_fp16), Llama-style prefill shapes
    if "fa" in which:
        res = {}
        for (T, nkv, dh, nh, nkvh, masked) in [(4096, 4096, 128, 32, 8, True), (4096, 4096, 128, 32, 8, False),
                                              (2048, 2048, 256, 16, 8, True)]:
            gf = torch.Generator(device="cuda")
            gf.manual_seed(T + dh)
            Qf = (torch.randn((nh, T, dh), device="cuda", generator=gf) * 0.5).half()
            Kf = (torch.randn((nkvh, nkv, dh), device="cuda", generator=gf) * 0.5).half()
            Vf = torch.randn((nkvh, dh, nkv), device="cuda", generator=gf).half()
            Mf = None
            if masked:
                pos = nkv - T + torch.arange(T, device="cuda")[:, None]
                Mf = torch.where(torch.arange(nkv, device="cuda")[None, :] <= pos, 0.0, float("-inf")).half()
            Of = torch.empty((nh, T, dh), device="cuda", dtype=torch.float16)
            runf = (lambda Qf=Qf, Kf=Kf, Vf=Vf, Mf=Mf, Of=Of, T=T, nkv=nkv, dh=dh, nh=nh, nkvh=nkvh:
                    L.rocket_flash_attn_fp16(dev.fd, T, nkv, dh, dh, nh, nkvh, dh ** -0.5, 0.0, Qf.data_ptr(),
                                             Kf.data_ptr(), Vf.data_ptr(),
                                             Mf.data_ptr() if Mf is not None else None, Of.data_ptr()))
            msf = timed(runf, 10)
            res[f"T{T}_kv{nkv}_dh{dh}_h{nh}/{nkvh}_{'causal' if masked else 'nomask'}"] = {
                "us": msf * 1e3, "tflops_all_scores": 4.0 * T * nkv * dh * nh / msf / 1e9}
        out["flash_attn_gqa"] = res

    # config 1: int8 64x512x256 one-shot (latency)
    if "c1" in which:
        import numpy as np
        A = np.random.default_rng(0).integers(-128, 128, (64, 512), dtype=np.int8)
        B = np.random.default_rng(1).integers(-128, 128, (256, 512), dtype=np.int8)
        C = np.zeros((64, 256), np.int32)
        dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
        dC = torch.empty((64, 256), dtype=torch.int32, device="cuda")
        t0 = time.perf_counter()
        for _ in range(200):
            dev.matmul_int8(64, 512, 256, dA, dB, dC)
        dev_us = (time.perf_counter() - t0) / 200 * 1e6
        t0 = time.perf_counter()
        for _ in range(200):
            dev.matmul_int8(64, 512, 256, A, B, C)
        host_us = (time.perf_counter() - t0) / 200 * 1e6
        exact = bool((C == (A.astype(np.int64) @ B.astype(np.int64).T).astype(np.int32)).all())
        out["config1_int8_latency"] = {"us_per_call_device_ptrs": dev_us, "us_per_call_host_ptrs": host_us,
                                       "bit_exact": exact,
                                       "note": "16.8 MOP: latency-bound, TOPS not meaningful"}
    dev.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true")
    ap.add_argument("--side", default="", help="comma list of side configs to run (c1,c2,c3,c4,ops,fa)")
    ap.add_argument("--side-only", action="store_true", help="run only the side configs (profiling)")
    ap.add_argument("--streams", type=int, default=4,
                    help="4: each GEMM of the set on its own context/stream (concurrent); 1: one stream")
    ap.add_argument("--layers", default="", help="comma list of GEMMs to run (profiling); default all four")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.side_only:
        import torch
        torch.cuda.set_device(0)
        rkb = load_pkg()
        peaks, _ = load_peaks()
        res = other_configs(rkb, torch, peaks, 2.0 * peaks.get("bf16_tflops", 1590.0),
                            tuple(args.side.split(",")) if args.side else ("c1", "c2", "c3", "c4", "ops", "fa"))
        print(json.dumps({"side_configs": res}), flush=True)
        return 0
    return main_ours(args)


if __name__ == "__main__":
    sys.exit(main())
