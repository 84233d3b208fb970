#!/usr/bin/env python
"""Benchmark of the LNS16 mul_mat hot path (G-LNSadd/s), one JSON line.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--mode base]
                    [--workload configs0|configs1]

Headline workload (default configs0): BASELINE configs[0], the case the
metric is quoted on ("@K=1536") -- weights 576 x 1536 (ggml src0
ne=(1536,576)), activations 1536 x 8 (src1 ne=(1536,8)), xlns16 codes
converted from numpy default_rng(0) N(0,0.02) / N(0,1) values; dst 8 x 576
xlns16 codes.  One step = one lnsb_mul_mat_lns call (the whole op, every
chain in element order).  configs1 (BASELINE configs[1]'s mul_mat, 1536 x 576
by 576 x 512) is reported beside it, and can be the headline instead.

Beside the headline: configs[1] with its own roofline, MUL_MAT_ID, the typed
weight decode, configs[1]'s normalisers against their chain bounds, the
configs[4] sweep points (8192 x 14336, N in {1, 16, 128}, sum32, output rows
split across the GPUs) and the model decodes of configs[2] / configs[3].

N > 1 (torchrun): weak scaling of the headline by output-row sharding -- each
rank owns its own weight rows of a (M * N)-row matrix, computes its shard,
and the step ends with the all-gather of the output shards fused into the
mul_mat's store (peer-memory stores over NVLink into two gather buffers used
by step parity, then a bounded peer-flag barrier).  configs[4] is strong
scaling: its 8192 rows are split N ways, gathered the same way.

--impl reference: the reference's CPU algorithm (the oracle restatement under
oracle/, the reference itself cannot be built: its arithmetic library is
absent) timed on this host's cores on the same workload.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "xlns-ggml-backend_b200"))

METRIC = "LNS16 mul_mat G-LNSadd/s"
UNIT = "G-LNSadd/s"
WORKLOADS = {
    "configs0": dict(desc="BASELINE configs[0] LNS16 mul_mat (K=1536): W 576x1536 x X 1536x8 -> 8x576 codes",
                     K=1536, M=576, N=8, seed=0),
    "configs1": dict(desc="BASELINE configs[1] LNS16 mul_mat: W 1536x576 (k-major codes) x X 576x512 -> 512x1536 codes",
                     K=576, M=1536, N=512, seed=1),
}
# Primitive integer operations of one LNS addition (including the operand
# product and the table load) in this build's restated algorithm, fixed per
# mode before tuning: the c_mode of the integer-issue roofline.
C_MODE = {"base": 18, "monte": 23, "monte_bylpvip": 34, "lpvip": 30, "sum32": 32}
SMS = 148
LANES_PER_SM = 128


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--mode", default="base", help="sum mode library of the headline (default base)")
    p.add_argument("--workload", default="configs0", choices=sorted(WORKLOADS))
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-decode", action="store_true", help="skip the model decode measurements")
    p.add_argument("--no-sides", action="store_true", help="the headline only (no side objects)")
    p.add_argument("--sides", default="all",
                   help="comma-separated side objects to run (configs, configs4, mul_mat_id, weights, normalisers, matvec; "
                        "default all) -- for profiling one of them")
    p.add_argument("--c4-points", default="1,16,128", help="configs[4] token counts N to time (default 1,16,128)")
    p.add_argument("--decode-mode", default="sum32", help="sum mode of the decode (BASELINE configs[2]: sum32)")
    p.add_argument("--decode-tokens", type=int, default=128,
                   help="tokens generated per sequence (BASELINE configs[2]: 128); fewer only for profiling")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("sm_max_mhz", 1965.0), "measured"
    except OSError:
        return 6650.0, 1965.0, "fallback"


# ncu capture summary of the kernel each (workload, mode) runs (DRAM bytes of one launch)
PROFILE = {
    ("configs0", "base"): "profiles/k_mul_mat16_res2_configs0.md",
    ("configs1", "base"): "profiles/k_mul_mat16_fast4_configs1.md",
    ("configs1", "monte"): "profiles/k_mul_mat16_fast_monte_configs1.md",
    ("configs1", "sum32"): "profiles/k_mul_mat_a32_sum32_configs1.md",
    ("configs1", "lpvip"): "profiles/k_mul_mat_a32_lpvip_configs1.md",
    ("configs1", "monte_bylpvip"): "profiles/k_mul_mat_a32_monte_bylpvip_configs1.md",
}


def traffic_of(key):
    try:
        with open(os.path.join(ROOT, PROFILE[key])) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except (OSError, KeyError, ValueError):
        pass
    return None


def adds_of(K, M, N):
    return M * N * max(K - 1, 0)


def algorithmic_bytes(K, M, N):
    return 2 * (K * M + K * N + M * N)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples during the timed region (read-only queries)."""
    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.bus = (bus_id or "").lower()
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and (not self.bus or self.bus.endswith(parts[0].lower()[-12:]) or parts[0].lower().endswith(self.bus[-12:])):
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------ CPU baseline (the checker's port)

def cpu_leg(wl, mode, seconds, nthreads):
    """Times the oracle's mul_mat (the reference algorithm restated in C) on the
    workload: the whole op, repeated to about `seconds`, or its first R weight
    rows against every token where one op takes longer than that."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle
    K, M, N = wl["K"], wl["M"], wl["N"]
    rng = np.random.default_rng(wl["seed"])
    w = oracle.from_f32_16(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    x = oracle.from_f32_16(rng.normal(0, 1, (N, K)).astype(np.float32))
    rows = max(1, min(M, 8))
    t0 = time.perf_counter()
    oracle.mul_mat16(mode, w[:rows], x, nthreads=nthreads)
    dt = time.perf_counter() - t0
    rows = int(max(1, min(M, rows * seconds / max(dt, 1e-6))))
    reps = 1
    if rows == M:
        t0 = time.perf_counter()
        oracle.mul_mat16(mode, w, x, nthreads=nthreads)
        reps = max(1, int(seconds / max(time.perf_counter() - t0, 1e-6)))
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle.mul_mat16(mode, w[:rows], x, nthreads=nthreads)
    dt = time.perf_counter() - t0
    adds = adds_of(K, rows, N) * reps
    what = ("the whole op x %d" % reps) if rows == M else ("first %d of %d weight rows x all %d tokens" % (rows, M, N))
    return {"value": adds / dt / 1e9, "unit": UNIT, "cores": nthreads, "kind": "port",
            "sample": "%s, K=%d (%d LNS adds, %.1f s)" % (what, K, adds, dt)}


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    nthreads = os.cpu_count() or 1
    vals = []
    for _ in range(args.warmup):
        cpu_leg(wl, args.mode, 0.3, nthreads)
    t0 = time.perf_counter()
    leg = None
    for _ in range(args.steps):
        leg = cpu_leg(wl, args.mode, 3.0, nthreads)
        vals.append(leg["value"])
    wall = time.perf_counter() - t0
    v = statistics.median(vals)
    leg["value"] = v
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": wall * 1000 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u16 (xlns16 codes)", "data": "synthetic",
        "config": {"workload": wl["desc"], "mode": args.mode, "sample": "per step: " + leg["sample"]},
        "cpu_baseline": leg, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


# ------------------------------------------------------------------ GPU helpers

class Ctx:
    """Per-process state: the rank, the process group, the L2 flush buffer,
    the stream and (N > 1) the peer-flag barrier of the fused all-gathers,
    whose epoch counts every barrier of the run (all ranks take the same
    steps in the same order)."""

    def __init__(self, torch, dist, rank, world):
        self.torch, self.dist, self.rank, self.world = torch, dist, rank, world
        self.flush = torch.empty(64 * 1024 * 1024, dtype=torch.int32, device="cuda")   # 256 MB > L2 (126 MB)
        self.stream = torch.cuda.current_stream()
        self.sp = ctypes.c_void_p(self.stream.cuda_stream)
        self.epoch = 0
        self.launches = 0
        if world > 1:
            import torch.distributed._symmetric_memory as symm_mem
            self.symm = symm_mem
            self.fbuf = symm_mem.empty(world, dtype=torch.int32, device="cuda")
            self.fbuf.zero_()
            self.fhdl = symm_mem.rendezvous(self.fbuf, dist.group.WORLD)
            self.berr = torch.zeros(1, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            dist.barrier()

    def barrier(self, lib):
        self.epoch += 1
        return lib.lnsb_group_barrier(ctypes.c_void_p(self.fhdl.buffer_ptrs_dev), self.world, self.rank, self.epoch,
                                      ctypes.c_void_p(self.berr.data_ptr()), self.sp)

    def check_barrier(self):
        if self.world > 1 and self.berr.item() != 0:
            raise SystemExit("peer barrier timed out")

    def max_over_ranks(self, *vals):
        if self.world == 1:
            return list(vals)
        t = self.torch.tensor(list(vals), dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.tolist()


class FusedGather:
    """Two symmetric-memory gather buffers of [N][M * world] codes used by step
    parity (the write-after-read rule of lnsb_mul_mat_lns_peers: each step's
    result is read on this rank's stream before its next call)."""

    def __init__(self, ctx, lib, fmt, N, M):
        torch = ctx.torch
        dt = torch.int16 if fmt == 16 else torch.int32
        self.ctx, self.lib, self.fmt, self.N, self.M = ctx, lib, fmt, N, M
        self.bufs = [ctx.symm.empty(N * M * ctx.world, dtype=dt, device="cuda") for _ in range(2)]
        for b in self.bufs:
            b.fill_(-1)
        self.hdls = [ctx.symm.rendezvous(b, ctx.dist.group.WORLD) for b in self.bufs]
        import lnsb200
        self.peers = [lnsb200._lib.PeerOut(h.buffer_ptrs_dev, ctx.world, M * ctx.world, ctx.rank * M) for h in self.hdls]
        self.i = 0
        torch.cuda.synchronize()
        ctx.dist.barrier()

    def step(self, argp, status):
        """one mul_mat with the gather fused into its store, then the barrier;
        returns the buffer that holds the gathered result"""
        b = self.i % 2
        self.i += 1
        st = self.lib.lnsb_mul_mat_lns_peers(self.fmt, argp, ctypes.byref(self.peers[b]), self.ctx.sp)
        st2 = self.ctx.barrier(self.lib)
        if st != 0 or st2 != 0:
            status[0] = st or st2
        self.ctx.launches += 2
        return self.bufs[b]


def timed(ctx, fn, steps, warmup, flush=True):
    """device time of `steps` calls of fn (ms, list), L2 flushed before each,
    after `warmup` untimed calls; max over ranks of the total"""
    torch = ctx.torch
    for _ in range(warmup):
        if flush:
            ctx.flush.zero_()
        fn()
    torch.cuda.synchronize()
    if ctx.dist:
        ctx.dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        if flush:
            ctx.flush.zero_()
        ev[i][0].record(ctx.stream)
        fn()
        ev[i][1].record(ctx.stream)
    torch.cuda.synchronize()
    ms = [b.elapsed_time(e) for b, e in ev]
    total, = ctx.max_over_ranks(sum(ms))
    return total / steps


def lns_operands(torch, np, ks, K, M, N, seed, rank=0):
    rng = np.random.default_rng(seed + 1000 * rank)
    w_f32 = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32)).cuda()    # ggml src0 rows
    x_f32 = torch.from_numpy(rng.normal(0, 1, (N, K)).astype(np.float32)).cuda()
    w = torch.empty(K * M, dtype=torch.int16, device="cuda")                          # k-major codes
    x = torch.empty(N * K, dtype=torch.int16, device="cuda")
    ks.to_lns_transposed(w_f32, w, M, K, M)
    ks.to_lns(x_f32, x)
    return w, x, rng


# ------------------------------------------------------------------ the headline

def run_ours(args, wl):
    import numpy as np
    import torch
    import lnsb200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    ctx = Ctx(torch, dist, rank, world)

    K, M, N = wl["K"], wl["M"], wl["N"]
    ks = lnsb200.KernelSet(16, args.mode)
    ks.upload_tables()
    lib = ks.lib
    w, x, rng = lns_operands(torch, np, ks, K, M, N, wl["seed"], rank)
    out = torch.empty(N * M, dtype=torch.int16, device="cuda")
    # the timed call goes straight to the C ABI with prebuilt arguments, so
    # host-side Python work cannot open gaps inside the event-timed region
    mm_args = lnsb200.MulMatArgs(w.data_ptr(), x.data_ptr(), None, K, M, N, 1, 1, 1, 1, 7)
    mm_argp = ctypes.byref(mm_args)
    out_p = ctypes.c_void_p(out.data_ptr())
    status = [0]

    gather = None
    if world > 1:
        from lnsb200 import shard
        gather = FusedGather(ctx, lib, 16, N, M)
        # the fused gather must give what NCCL's does, bit for bit, on two steps
        for _ in range(2):
            g = gather.step(mm_argp, status)
            lib.lnsb_mul_mat_lns(16, mm_argp, out_p, ctx.sp)
            want = shard.all_gather_rows(out.view(N, M), world).contiguous().view(-1)
            torch.cuda.synchronize()
            ctx.check_barrier()
            if not torch.equal(g, want):
                raise SystemExit("fused peer all-gather differs from the NCCL all-gather")

    def step():
        if gather is not None:
            gather.step(mm_argp, status)
        else:
            st = lib.lnsb_mul_mat_lns(16, mm_argp, out_p, ctx.sp)
            if st != 0:
                status[0] = st
            ctx.launches += 1

    bus = None
    try:
        p = torch.cuda.get_device_properties(local)
        bus = "%02x:%02x.0" % (p.pci_bus_id, p.pci_device_id)
    except Exception:
        pass
    # the launch count of the timed region: this step's kernels only
    sampler = ClockSampler(bus)
    sampler.start()
    time.sleep(0.4)
    for _ in range(args.warmup):
        ctx.flush.zero_()
        step()
    torch.cuda.synchronize()
    ctx.launches = 0
    step_ms = timed(ctx, step, args.steps, 0)
    launches = ctx.launches
    clocks = sampler.stop()
    if status[0] != 0:
        raise lnsb200.LnsbError(lib, "lnsb_mul_mat_lns", status[0])
    ctx.check_barrier()
    # the mul_mat alone (N > 1: without its gather stores and barrier)
    kern_ms = step_ms if world == 1 else timed(ctx, lambda: lib.lnsb_mul_mat_lns(16, mm_argp, out_p, ctx.sp), args.steps, 2)

    e2e_ms, h2d, d2h = e2e_run(ctx, ks, w, rng, K, M, N, gather, mm_args, args)

    adds = adds_of(K, M, N)
    value = adds * world / (step_ms / 1000) / 1e9
    e2e_val = adds * world / (e2e_ms / 1000) / 1e9
    hbm, smmax, src = peaks()
    f_mhz = clocks.get("sm_mhz") or smmax
    c = C_MODE.get(args.mode, 18)
    int_peak = SMS * LANES_PER_SM * f_mhz * 1e6 / c / 1e9
    kern_s = kern_ms / 1000
    achieved = adds / kern_s / 1e9
    bytes_alg = algorithmic_bytes(K, M, N)
    roof = {"bound": "int", "achieved": achieved, "peak": int_peak, "unit": UNIT, "frac": achieved / int_peak,
            "traffic": traffic_of((args.workload, args.mode)), "traffic_source": PROFILE.get((args.workload, args.mode)),
            "c_mode": c, "sm_mhz_used": f_mhz,
            "note": "integer-issue bound: %d SMs x %d lanes x f_sm / c_mode (%s SM clock)" % (
                SMS, LANES_PER_SM, "sampled" if clocks.get("sm_mhz") else src),
            "hbm": {"achieved_gbs": bytes_alg / kern_s / 1e9, "peak_gbs": hbm, "frac": bytes_alg / kern_s / 1e9 / hbm,
                    "algorithmic_bytes": bytes_alg}}
    if args.mode == "base" and args.workload == "configs0":
        # the chain bound: K - 1 dependent additions per output, every output in
        # parallel; L_add measured live on this GPU (lnsb_add_latency, key form, 16
        # distinct chains per warp as the latency kernel runs configs[0])
        l_add = ks.add_latency(0, 16, 4096)
        t_chain = (K - 1) * l_add / (f_mhz * 1e6)
        roof["chain"] = {"l_add_cycles": l_add, "lanes": 16, "t_chain_us": t_chain * 1e6, "kernel_us": kern_ms * 1000,
                         "frac": t_chain / kern_s,
                         "note": "diagnostic bound T_chain = (K-1) L_add / f_sm; the event-timed kernel includes its launch"}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u16 (xlns16 codes; integer LNS arithmetic)", "data": "synthetic",
        "config": {"workload": wl["desc"] + (" per rank, output rows sharded + fused all-gather" if world > 1 else ""),
                   "K": K, "M": M, "N": N, "mode": args.mode, "parallelism": "rowshard%d" % world,
                   "gather": ("fused into the mul_mat store: peer-memory stores over NVLink into two gather buffers "
                              "by step parity + a bounded peer-flag barrier (checked bit for bit against NCCL)")
                   if world > 1 else None,
                   "l2": "flushed (256 MB write) before every timed step"},
        "roofline": roof,
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "per step: H2D of F32 activations (pinned), " +
                        ("lnsb_mul_mat_xf32 (the activations' conversion and mul_mat in one call, F32 out)"
                         if world == 1 else
                         "lnsb_to_lns, lnsb_mul_mat_lns_peers + lnsb_group_barrier (the fused all-gather), "
                         "lnsb_to_f32 of the gathered codes") +
                        ", D2H of the F32 result (pinned); double buffered, copies on their own streams",
                "l2": "not flushed between steps: a serving loop's steady state, weights resident (value flushes)"},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if not args.no_sides:
        sides = set(args.sides.split(",")) if args.sides != "all" else \
            {"configs", "configs4", "mul_mat_id", "weights", "normalisers", "matvec"}
        other = "configs1" if args.workload == "configs0" else "configs0"
        if "configs" in sides:
            line[other] = time_side_mul_mat(ctx, lnsb200, torch, np, WORKLOADS[other], args, int_peak, f_mhz)
        if "configs4" in sides:
            line["configs4"] = time_configs4(ctx, lnsb200, torch, np, args, f_mhz)
        if world == 1:
            if "mul_mat_id" in sides:
                line["mul_mat_id"] = time_mul_mat_id(ctx, lnsb200, torch, np, args, int_peak)
            if "weights" in sides:
                line["weights"] = time_weights(ctx, lnsb200, torch, np, args, hbm)
            if "normalisers" in sides:
                line["normalisers"] = time_norms(ctx, lnsb200, torch, np, args, f_mhz)
            if "matvec" in sides:
                line["matvec"] = time_matvec(ctx, lnsb200, torch, np, args, f_mhz)
    if not args.no_decode:
        # the metric's second half: model decode tok/s, one sequence per GPU
        line["decode"] = run_decode(torch, dist, rank, world, args, cpu=(rank == 0 and world == 1 and not args.no_cpu_baseline),
                                    f_mhz=f_mhz)
        if world == 1:
            # the same model and prompt in LNS32, on 1 GPU
            line["decode_lns32"] = run_decode(torch, dist, rank, world, args,
                                              cpu=(rank == 0 and not args.no_cpu_baseline), fmt=32, f_mhz=f_mhz)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_leg(wl, args.mode, 10.0, os.cpu_count() or 1)
        # the reference's CPU backend runs one thread (its ops are sequential loops): the
        # same port on one core, beside the all-cores figure, and the GPU's ratio to each
        st = cpu_leg(wl, args.mode, 5.0, 1)
        line["cpu_baseline"]["single_thread"] = st
        line["cpu_baseline"]["gpu_ratio"] = {"all_cores": value / line["cpu_baseline"]["value"],
                                             "single_thread": value / st["value"],
                                             "e2e_all_cores": e2e_val / line["cpu_baseline"]["value"],
                                             "e2e_single_thread": e2e_val / st["value"]}
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def e2e_run(ctx, ks, w, rng, K, M, N, gather, mm_args, args):
    """End to end through the C ABI with host buffers: every step uploads its
    F32 activations from pinned host memory (H2D), converts them and runs
    mul_mat -- on one GPU in one call (lnsb_mul_mat_xf32), at N > 1 to_lns and
    mul_mat with the fused all-gather and its barrier, then the gathered
    codes' decode (to_f32) -- and reads the F32 result back into
    pinned host memory (D2H); the weights stay resident, as the reference's
    weight cache keeps them.  Steps are double buffered the way a serving
    loop runs them: step i+1's upload and step i's read-back go on their own
    copy streams, so the copies overlap the kernels of the neighbouring
    steps.  Returns (ms per step, max over ranks; H2D bytes; D2H bytes)."""
    import numpy as np
    torch = ctx.torch
    import lnsb200
    NB, world = 2, ctx.world
    MO = M * world
    xh = torch.from_numpy(rng.normal(0, 1, (N, K)).astype(np.float32)).pin_memory()
    yh = [torch.empty(N * MO, dtype=torch.float32).pin_memory() for _ in range(NB)]
    xd = [torch.empty(N * K, dtype=torch.float32, device="cuda") for _ in range(NB)]
    xc = [torch.empty(N * K, dtype=torch.int16, device="cuda") for _ in range(NB)]
    yd = [torch.empty(N * MO, dtype=torch.float32, device="cuda") for _ in range(NB)]
    # one GPU: the F32 activations go straight to lnsb_mul_mat_xf32 (xc[b] its
    # x_work); with the gather, to_lns into xc[b] and the peer-store mul_mat
    args_b = [lnsb200.MulMatArgs(w.data_ptr(), (xd[b] if gather is None else xc[b]).data_ptr(), yd[b].data_ptr(),
                                 K, M, N, 1, 1, 1, 1, 7) for b in range(NB)]
    stream = ctx.stream
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_up = [torch.cuda.Event() for _ in range(NB)]        # input b uploaded
    ev_cv = [torch.cuda.Event() for _ in range(NB)]        # input b converted: xd[b] free
    ev_mm = [torch.cuda.Event() for _ in range(NB)]        # result b computed
    ev_dn = [torch.cuda.Event() for _ in range(NB)]        # result b read back: yd[b] free
    status = [0]

    def upload(i):
        b = i % NB
        up.wait_event(ev_cv[b])
        with torch.cuda.stream(up):
            xd[b].copy_(xh.view(-1), non_blocking=True)
        ev_up[b].record(up)

    def compute(i):
        b = i % NB
        stream.wait_event(ev_up[b])
        stream.wait_event(ev_dn[b])
        if gather is None:
            st = ks.lib.lnsb_mul_mat_xf32(16, ctypes.byref(args_b[b]), ctypes.c_void_p(xc[b].data_ptr()), ctx.sp)
            if st != 0:
                raise lnsb200.LnsbError(ks.lib, "lnsb_mul_mat_xf32", st)
            ev_cv[b].record(stream)
        else:
            ks.to_lns(xd[b], xc[b], stream=stream)
            ev_cv[b].record(stream)
            g = gather.step(ctypes.byref(args_b[b]), status)
            ks.to_f32(g, yd[b], stream=stream)             # the read of this step's gather, on this stream
        ev_mm[b].record(stream)

    def download(i):
        b = i % NB
        down.wait_event(ev_mm[b])
        with torch.cuda.stream(down):
            yh[b].copy_(yd[b], non_blocking=True)
        ev_dn[b].record(down)

    def run(n):
        up.wait_stream(stream)
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)
            download(i)
        stream.wait_event(ev_dn[(n - 1) % NB])

    run(max(3, args.warmup))
    torch.cuda.synchronize()
    if ctx.dist:
        ctx.dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    if status[0] != 0:
        raise lnsb200.LnsbError(ks.lib, "lnsb_mul_mat_lns_peers", status[0])
    ctx.check_barrier()
    ms, = ctx.max_over_ranks(e0.elapsed_time(e1))
    if ctx.dist:
        ctx.dist.barrier()
    return ms / args.steps, N * K * 4, N * MO * 4


# ------------------------------------------------------------------ side objects

def time_side_mul_mat(ctx, lnsb200, torch, np, wl, args, int_peak, f_mhz):
    """Another BASELINE mul_mat workload through the same C ABI call (inputs
    resident, L2 flushed before every step; N > 1: this rank's rows with the
    fused all-gather), with its roofline."""
    K, M, N = wl["K"], wl["M"], wl["N"]
    ks = lnsb200.KernelSet(16, args.mode)
    lib = ks.lib
    w, x, _ = lns_operands(torch, np, ks, K, M, N, wl["seed"], ctx.rank)
    out = torch.empty(N * M, dtype=torch.int16, device="cuda")
    a = lnsb200.MulMatArgs(w.data_ptr(), x.data_ptr(), None, K, M, N, 1, 1, 1, 1, 7)
    ap, op = ctypes.byref(a), ctypes.c_void_p(out.data_ptr())
    status = [0]
    gather = FusedGather(ctx, lib, 16, N, M) if ctx.world > 1 else None

    def call():
        if gather is not None:
            gather.step(ap, status)
        elif lib.lnsb_mul_mat_lns(16, ap, op, ctx.sp) != 0:
            status[0] = -1
    ms = timed(ctx, call, max(args.steps, 20), args.warmup)
    if status[0] != 0:
        raise RuntimeError("lnsb_mul_mat_lns failed on %s" % wl["desc"])
    ctx.check_barrier()
    adds = adds_of(K, M, N) * ctx.world
    val = adds / (ms / 1000) / 1e9
    c = C_MODE.get(args.mode, 18)
    out_d = {"workload": wl["desc"] + (" per rank, fused all-gather" if ctx.world > 1 else ""), "mode": args.mode,
             "ms_per_step": ms, "value": val, "unit": UNIT,
             "roofline": {"bound": "int", "achieved": val / ctx.world, "peak": int_peak, "frac": val / ctx.world / int_peak,
                          "unit": UNIT, "c_mode": c, "traffic": traffic_of((wl_key(wl), args.mode)),
                          "traffic_source": PROFILE.get((wl_key(wl), args.mode))},
             "l2": "flushed (256 MB write) before every timed step"}
    if args.mode == "base" and wl_key(wl) == "configs0":
        l_add = ks.add_latency(0, 16, 4096)
        t_chain = (K - 1) * l_add / (f_mhz * 1e6)
        out_d["roofline"]["chain"] = {"l_add_cycles": l_add, "t_chain_us": t_chain * 1e6, "frac": t_chain / (ms / 1000)}
    return out_d


def wl_key(wl):
    for k, v in WORKLOADS.items():
        if v is wl:
            return k
    return None


def time_configs4(ctx, lnsb200, torch, np, args, f_mhz):
    """BASELINE configs[4] sweep points (sum32): W 8192 x 14336 N(0,0.02), X
    14336 x N N(0,1), N in {1, 16, 128}; the 8192 output rows split into
    ctx.world contiguous blocks (strong scaling), each rank's block gathered
    on every GPU by the fused peer-store all-gather.  Weights are generated on
    the device per 1024-row block (torch generator seeded 3000 + block), so
    every GPU count runs the same matrix; activations numpy default_rng(3)."""
    K, MT = 14336, 8192
    world, rank = ctx.world, ctx.rank
    Mr = MT // world
    ks = lnsb200.KernelSet(16, "sum32")
    ks.upload_tables()
    lib = ks.lib
    w = torch.empty(K * Mr, dtype=torch.int16, device="cuda")
    blk = 1024
    wf = torch.empty((blk, K), dtype=torch.float32, device="cuda")
    for b in range(Mr // blk):
        g = torch.Generator(device="cuda")
        g.manual_seed(3000 + rank * (Mr // blk) + b)
        wf.normal_(0.0, 0.02, generator=g)
        ks.to_lns_transposed(wf, w[b * blk:], blk, K, Mr)
    del wf
    res = {}
    for N in (int(n) for n in args.c4_points.split(",")):
        xf = torch.from_numpy(np.random.default_rng(3).normal(0, 1, (N, K)).astype(np.float32)).cuda()
        x = torch.empty(N * K, dtype=torch.int16, device="cuda")
        ks.to_lns(xf, x)
        out = torch.empty(N * Mr, dtype=torch.int16, device="cuda")
        a = lnsb200.MulMatArgs(w.data_ptr(), x.data_ptr(), None, K, Mr, N, 1, 1, 1, 1, 7)
        ap, op = ctypes.byref(a), ctypes.c_void_p(out.data_ptr())
        status = [0]
        gather = FusedGather(ctx, lib, 16, N, Mr) if world > 1 else None
        if gather is not None:
            from lnsb200 import shard
            g = gather.step(ap, status)
            lib.lnsb_mul_mat_lns(16, ap, op, ctx.sp)
            want = shard.all_gather_rows(out.view(N, Mr), world).contiguous().view(-1)
            torch.cuda.synchronize()
            ctx.check_barrier()
            if not torch.equal(g, want):
                raise SystemExit("configs4: fused peer all-gather differs from the NCCL all-gather")

        def call():
            if gather is not None:
                gather.step(ap, status)
            elif lib.lnsb_mul_mat_lns(16, ap, op, ctx.sp) != 0:
                status[0] = -1
        steps = 3 if N == 128 else 6
        ms = timed(ctx, call, steps, 2)
        if status[0] != 0:
            raise RuntimeError("configs4 mul_mat failed")
        ctx.check_barrier()
        adds = adds_of(K, MT, N)
        int_peak = SMS * LANES_PER_SM * f_mhz * 1e6 / C_MODE["sum32"] / 1e9
        val = adds / (ms / 1000) / 1e9
        res["N%d" % N] = {"ms_per_step": ms, "value": val, "unit": UNIT, "adds": adds,
                          "frac_int": val / world / int_peak,
                          "bound": "chain latency (K dependent sum32 additions)" if N == 1 else "integer issue"}
        del gather
    return {"workload": "BASELINE configs[4] LNS16 sum32 mul_mat: W 8192x14336 x X 14336xN, rows split %d ways" % world,
            "mode": "sum32", "K": K, "rows_per_gpu": Mr, "scaling": "strong", "n_gpus": world, "points": res,
            "gather": "fused peer-store all-gather + barrier" if world > 1 else None,
            "l2": "flushed (256 MB write) before every timed step"}


def time_norms(ctx, lnsb200, torch, np, args, f_mhz):
    """BASELINE configs[1]'s normalisers on xlns16 codes, device-timed, L2
    flushed before every step: soft_max over logits N(0, 3) shaped [9 heads]
    [512 queries][512 keys] with a causal mask (keys after the query are
    -inf) and scale 1.0 (4,608 rows x 511 additions, masked zeros included),
    and rms_norm over 512 rows of 576 N(0, 1) values, eps 1e-5 (576 additions
    per row); inputs numpy default_rng(1), converted to codes on the device.
    Bound: one row's chain of dependent additions, every row in parallel:
    T_chain = additions per row x L_add / f_sm, L_add measured on this GPU
    (lnsb_add_latency: the non-negative addition the mode's normalisers run)."""
    ks = lnsb200.KernelSet(16, args.mode)
    lib = ks.lib
    rng = np.random.default_rng(1)
    n, q, h = 512, 512, 9
    logits = torch.from_numpy(rng.normal(0, 3, (h, q, n)).astype(np.float32)).cuda()
    sm_src = torch.empty(h * q * n, dtype=torch.int16, device="cuda")
    ks.to_lns(logits.view(-1), sm_src)
    mask_np = np.zeros((q, n), np.uint16)
    mask_np[np.triu_indices(q, 1, n)] = 0xFFFF                       # xlns16 -inf after the query
    mask = torch.from_numpy(mask_np.view(np.int16)).cuda()
    sm_dst = torch.empty_like(sm_src)
    sm_work = torch.empty_like(sm_src)
    rows, cols = 512, 576
    x = torch.from_numpy(rng.normal(0, 1, (rows, cols)).astype(np.float32)).cuda()
    rn_src = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
    ks.to_lns(x.view(-1), rn_src)
    rn_dst = torch.empty_like(rn_src)
    ne = (ctypes.c_int64 * 4)(n, q, h, 1)
    mne = (ctypes.c_int64 * 4)(n, q, 1, 1)
    sp = ctx.sp
    P = lambda t: ctypes.c_void_p(t.data_ptr())                        # noqa: E731
    kind = {"base": 1, "sum32": 2}.get(args.mode)
    l_add = ks.add_latency(kind, 32, 4096) if kind is not None else None
    calls = {
        "soft_max": (lambda: lib.lnsb_soft_max_lns(16, P(sm_src), ne, P(mask), mne, 0x4000, P(sm_dst), P(sm_work), 7, sp),
                     h * q * (n - 1), n - 1, h * q, "[9][512][512] xlns16 logits N(0,3), causal mask, scale 1.0"),
        "rms_norm": (lambda: lib.lnsb_rms_norm_lns(16, P(rn_src), P(rn_dst), cols, rows, ctypes.c_float(1e-5), 7, sp),
                     rows * cols, cols, rows, "512 x 576 xlns16 values N(0,1), eps 1e-5"),
    }
    out = {}
    for name, (call, adds, per_row, nrows, what) in calls.items():
        ms = timed(ctx, call, max(args.steps, 20), args.warmup)
        d = {"workload": "BASELINE configs[1] %s: %s" % (name, what), "mode": args.mode, "ms_per_step": ms,
             "value": adds / (ms / 1000) / 1e9, "unit": UNIT, "adds": adds,
             "bound": "chain latency: %d dependent additions per row, %d rows" % (per_row, nrows),
             "l2": "flushed (256 MB write) before every timed step"}
        if l_add is not None:
            t_chain = per_row * l_add / (f_mhz * 1e6)
            d["chain"] = {"l_add_cycles": l_add, "t_chain_us": t_chain * 1e6, "frac": t_chain / (ms / 1000),
                          "adder": "non-negative xlns16 (padd16)" if kind == 1 else "non-negative xlns32 (padd32f)"}
        out[name] = d
    return out


def time_matvec(ctx, lnsb200, torch, np, args, f_mhz):
    """The decode's mat-vecs (BASELINE configs[2] / [3] shapes, one token):
    q/k/v (576 -> 960), up/gate (576 -> 3072) and down (1536 -> 576) in LNS16
    sum32 and LNS32, weights N(0, 0.02), the token N(0, 1) (numpy
    default_rng(5)), codes in and out, device-timed, L2 flushed before every
    step.  Bound: the chain, K - 1 dependent additions per output through the
    general xlns32 adder, L_add measured on this GPU (lnsb_add_latency kind 3):
    T_chain = (K - 1) L_add / f_sm."""
    rng = np.random.default_rng(5)
    out = {}
    shapes = (("qkv", 576, 960), ("up_gate", 576, 3072), ("down", 1536, 576))
    for fmt, mode in ((16, "sum32"), (32, "base")):
        ks = lnsb200.KernelSet(fmt, mode)
        ks.upload_tables()
        l_add = ks.add_latency(3, 32, 4096)
        dt = torch.int16 if fmt == 16 else torch.int32
        for name, K, M in shapes:
            wf = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32)).cuda()
            xf = torch.from_numpy(rng.normal(0, 1, (1, K)).astype(np.float32)).cuda()
            w = torch.empty(K * M, dtype=dt, device="cuda")
            ks.to_lns_transposed(wf, w, M, K, M)
            x = torch.empty(K, dtype=dt, device="cuda")
            ks.to_lns(xf, x)
            y = torch.empty(M, dtype=dt, device="cuda")
            ms = timed(ctx, lambda: ks.mul_mat_lns(w, x, y, K, M, 1, stream=ctx.stream), max(args.steps, 20), args.warmup)
            t_chain = (K - 1) * l_add / (f_mhz * 1e6)
            out["%s_%s" % ("lns16_sum32" if fmt == 16 else "lns32", name)] = {
                "K": K, "M": M, "ms_per_step": ms, "value": M * (K - 1) / (ms / 1000) / 1e9, "unit": UNIT,
                "cycles_per_step": ms / 1000 * f_mhz * 1e6 / (K - 1),
                "chain": {"l_add_cycles": l_add, "t_chain_us": t_chain * 1e6, "frac": t_chain / (ms / 1000),
                          "adder": "general xlns32 (add32f_sel)"}}
    out["kernel"] = "k_mat_vec_lat: a producer warp writes the products into a shared ring, the chain warp adds"
    out["l2"] = "flushed (256 MB write) before every timed step"
    return out


def time_mul_mat_id(ctx, lnsb200, torch, np, args, int_peak):
    """MUL_MAT_ID on a mixture-of-experts FFN shape (8 experts of 1536 x 576,
    128 tokens, 2 experts per token; synthetic N(0,0.02) / N(0,1) codes, seed
    4), device-timed, L2 flushed before every step; roofline as the main
    line's (integer issue at the mode's c_mode)."""
    n_exp, K, M, n_tok, n_used = 8, 576, 1536, 128, 2
    ks = lnsb200.KernelSet(16, args.mode)
    rng = np.random.default_rng(4)
    w = torch.empty(n_exp * K * M, dtype=torch.int16, device="cuda")
    for e in range(n_exp):
        wf = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32)).cuda()
        ks.to_lns_transposed(wf, w[e * K * M:(e + 1) * K * M], M, K, M)
    xf = torch.from_numpy(rng.normal(0, 1, (n_tok, K)).astype(np.float32)).cuda()
    x = torch.empty(n_tok * K, dtype=torch.int16, device="cuda")
    ks.to_lns(xf, x)
    ids = torch.from_numpy(rng.integers(0, n_exp, (n_tok, n_used)).astype(np.int32)).cuda()
    out = torch.empty(n_tok * n_used * M, dtype=torch.int16, device="cuda")
    ms = timed(ctx, lambda: ks.mul_mat_id_lns(w, x, ids, out, K, M, n_exp, 1, n_used, n_tok, stream=ctx.stream),
               max(args.steps, 10), max(3, args.warmup))
    adds = n_tok * n_used * M * (K - 1)
    val = adds / (ms / 1000) / 1e9
    return {"workload": "MUL_MAT_ID: 8 experts of 1536x576, 128 tokens x 2 experts (synthetic, seed 4)",
            "mode": args.mode, "ms_per_step": ms, "value": val, "unit": UNIT,
            "roofline": {"bound": "int", "achieved": val, "peak": int_peak, "frac": val / int_peak, "unit": UNIT},
            "l2": "flushed (256 MB write) before every timed step"}


def time_weights(ctx, lnsb200, torch, np, args, hbm):
    """Weights in ggml storage types decoded on the device into the k-major LNS
    image (lnsb_to_lns_transposed_typed), 8192 x 4096 per type; algorithmic
    bytes = the packed rows read + the codes written; bound HBM."""
    ks = lnsb200.KernelSet(16, args.mode)
    rows, cols = 8192, 4096
    rng = np.random.default_rng(5)
    out = {}
    dst = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
    for t in ("f16", "q8_0", "q4_k", "q6_k"):
        rb = ks.type_row_bytes(t, cols)
        if t == "f16":
            raw = torch.from_numpy(rng.normal(0, 0.05, (rows, cols)).astype(np.float16).view(np.uint8)).cuda()
        else:
            # random quants under finite f16 block scales (1e-3 .. 1e-1), as a quantiser writes them
            qk, bb = {"q8_0": (32, 34), "q4_k": (256, 144), "q6_k": (256, 210)}[t]
            blocks = rng.integers(0, 256, (rows, cols // qk, bb), dtype=np.uint8)
            for off in {"q8_0": [0], "q4_k": [0, 2], "q6_k": [208]}[t]:
                d = rng.uniform(1e-3, 1e-1, (rows, cols // qk)).astype(np.float16)
                blocks[:, :, off:off + 2] = d.view(np.uint8).reshape(rows, cols // qk, 2)
            raw = torch.from_numpy(blocks.reshape(rows, rb)).cuda()
        ms = timed(ctx, lambda: ks.to_lns_transposed_typed(t, raw, dst, rows, cols, rows, stream=ctx.stream), 10, 3)
        by = rows * rb + rows * cols * 2
        out[t] = {"ms": ms, "gbs": by / (ms / 1000) / 1e9, "frac_hbm": by / (ms / 1000) / 1e9 / hbm, "bytes": by}
    return {"workload": "8192 x 4096 weight -> xlns16 k-major image, per storage type", "bound": "hbm",
            "peak_gbs": hbm, "types": out,
            "l2": "flushed (256 MB write) before every timed launch", "launches_per_type": 10}


def run_decode(torch, dist, rank, world, args, cpu=False, fmt=16, f_mhz=1965.0):
    """BASELINE configs[2] (fmt 16) and configs[3] (fmt 32): SmolLM2-135M-shaped
    random-init Llama, LNS16 in the decode sum mode or LNS32, 128-token prompt
    prefill then 128-token greedy decode, one independent sequence per GPU
    (prompt seed 2 + rank).  Device-timed with events; each step's token goes
    back to the host (greedy argmax) and the next token id comes from it, so
    the decode is end to end.  The time is the max over ranks; tok/s counts
    every rank's tokens."""
    import lnsb200.model as model
    cfg = model.SMOLLM2_135M
    w = model.init_weights(cfg, seed=2)
    g = model.GpuOps(cfg, w, mode=args.decode_mode, n_ctx=256, fmt=fmt)
    prompt = model.prompt_ids(cfg, 128, seed=2 + rank)
    stream = torch.cuda.current_stream()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    model.forward(g, cfg, prompt[:8], 0)                 # warm-up (also fills the allocator)
    dec = model.GraphDecoder(g, cfg)                     # one CUDA graph per decode position,
    G = args.decode_tokens - 1                          # steps after the prefill's token
    dec.prepare(len(prompt), len(prompt) + G)            # captured once before the timed region
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e[0].record(stream)
    logits = model.forward(g, cfg, prompt, 0)
    toks = [g.argmax(logits)]
    e[1].record(stream)
    toks += dec.decode(toks[0], len(prompt), G)         # each step's token copied to pinned host memory
    e[2].record(stream)
    torch.cuda.synchronize()
    pre_ms, dec_ms = e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])
    if dist:
        t = torch.tensor([pre_ms, dec_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre_ms, dec_ms = t.tolist()
    out = {"model": "SmolLM2-135M shape (30 layers, d 576, 9/3 heads, ffn 1536, vocab 49152), random N(0,0.02) weights seed 2",
           "format": "xlns%d" % fmt, "mode": args.decode_mode if fmt == 16 else None, "prompt": 128, "generated": G + 1, "sequences": world,
           "prefill_tok_per_s": world * 128 / (pre_ms / 1000), "decode_tok_per_s": world * G / (dec_ms / 1000),
           "ms_per_token": dec_ms / G, "prefill_ms": pre_ms,
           "timing": "device events; prefill eager, decode as one CUDA graph per position (captured before the timed region); each step's greedy token is copied to pinned host memory",
           "first_tokens": toks[:8]}
    # the chain bound of one decode step: its dependent additions, the general
    # xlns32 addition (mat-vecs, q.K and p.V chains) and the non-negative one
    # (rms_norm and softmax normalisers), at their measured latencies (sum32 and
    # xlns32 run both on the flat xlns32 adder)
    import lnsb200
    if fmt == 32 or args.decode_mode == "sum32":
        ks = lnsb200.KernelSet(fmt, args.decode_mode if fmt == 16 else "base")
        ks.upload_tables()
        l3, l2 = ks.add_latency(3, 32), ks.add_latency(2, 32)
        L, d, ffn, hd = cfg["n_layer"], cfg["n_embd"], cfg["n_ff"], cfg["head_dim"]
        nkv = (129 + 128 + G) / 2                         # keys per step, averaged over the G steps
        s3 = L * (d + hd + nkv + d + d + ffn) + d          # qkv, q.K, p.V, wo, up/gate, down; output
        s2 = L * (d + d + nkv - 1) + d                     # two norm blocks and the softmax per layer; final norm
        f = f_mhz * 1e6
        t_chain = (s3 * l3 + s2 * l2) / f * 1e3
        out["chain"] = {"general_steps": s3, "nonneg_steps": s2, "l_add_general_cycles": l3, "l_add_nonneg_cycles": l2,
                        "sm_mhz_used": f / 1e6, "t_chain_ms_per_token": t_chain, "frac": t_chain / (dec_ms / G),
                        "bound": "one token's dependent additions (mat-vec, attention and normaliser chains) at "
                                 "the measured latency of each adder"}
    if cpu:
        # the CPU oracle (the reference's algorithm, host cores) on a bounded sample:
        # prefill of 8 tokens, then 16 decode steps (a few seconds)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracle_model import OracleOps
        o = OracleOps(cfg, w, mode=args.decode_mode, n_ctx=32, nthreads=os.cpu_count() or 1, fmt=fmt)
        lo = model.forward(o, cfg, prompt[:8], 0)
        t0 = time.perf_counter()
        tk = o.argmax(lo)
        for p in range(8, 24):
            tk = o.argmax(model.forward(o, cfg, [tk], p))
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"decode_tok_per_s": 16 / dt, "cores": os.cpu_count() or 1, "kind": "port",
                               "sample": "oracle model: 8-token prefill, then 16 decode steps timed (%.1f s)" % dt}
    return out


def main():
    args = parse()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_ours(args, wl)


if __name__ == "__main__":
    sys.exit(main())
