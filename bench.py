#!/usr/bin/env python
"""Benchmark of the LNS16 mul_mat hot path (G-LNSadd/s), one JSON line.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--mode base]
                    [--workload configs1|configs0]

Workload (default configs1): BASELINE configs[1]'s mul_mat -- weights
1536 x 576 (ggml src0 ne=(576,1536)), activations 576 x 512 (src1 ne=(576,512)),
xlns16 codes converted from numpy default_rng(1) N(0,0.02) / N(0,1) values;
dst 512 x 1536 xlns16 codes.  One step = one lnsb_mul_mat_lns call (the whole
op, every chain in element order).  configs0 is the reference's own CPU case
(576 x 1536 by 1536 x 8, K = 1536).

N > 1 (torchrun): weak scaling by output-row sharding -- each rank owns 1536
different weight rows of a (1536 * N)-row matrix, computes its shard and the
step ends with an NCCL all-gather of the output shards (the exchange step).

--impl reference: the reference's CPU algorithm (the oracle restatement under
oracle/, the reference itself cannot be built: its arithmetic library is
absent) timed on this host's cores on a bounded sample of the same workload.
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
    "configs1": dict(desc="BASELINE configs[1] LNS16 mul_mat: W 1536x576 (k-major codes) x X 576x512 -> 512x1536 codes",
                     K=576, M=1536, N=512, seed=1),
    "configs0": dict(desc="BASELINE configs[0] LNS16 mul_mat: W 576x1536 x X 1536x8 -> 8x576 codes",
                     K=1536, M=576, N=8, seed=0),
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
    p.add_argument("--mode", default=None, help="sum mode library (default: base; sum32 for configs4)")
    p.add_argument("--workload", default="configs1", choices=sorted(WORKLOADS) + ["configs4"])
    p.add_argument("--sweep-k", type=int, default=4096, help="configs4: K in {2048, 4096, 8192, 14336}")
    p.add_argument("--sweep-n", type=int, default=16, help="configs4: tokens in {1, 16, 128}")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-decode", action="store_true", help="skip the model decode measurement")
    p.add_argument("--decode-mode", default="sum32", help="sum mode of the decode (BASELINE configs[2]: sum32)")
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
    ("configs1", "base"): "profiles/k_mul_mat16_fast4_configs1.md",
    ("configs0", "base"): "profiles/k_mul_mat16_res_configs0.md",
    ("configs1", "monte"): "profiles/k_mul_mat16_fast_monte_configs1.md",
    ("configs1", "sum32"): "profiles/k_mul_mat_a32_sum32_configs1.md",
    ("configs1", "lpvip"): "profiles/k_mul_mat_a32_lpvip_configs1.md",
    ("configs1", "monte_bylpvip"): "profiles/k_mul_mat_a32_monte_bylpvip_configs1.md",
    ("configs4:4096:16", "sum32"): "profiles/k_mul_mat_a32_sum32_configs4_K4096_N16.md",
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
    """Times the oracle's mul_mat (the reference algorithm restated in C) on a
    bounded sample of the workload: the first R weight rows against all tokens."""
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
    t0 = time.perf_counter()
    oracle.mul_mat16(mode, w[:rows], x, nthreads=nthreads)
    dt = time.perf_counter() - t0
    adds = adds_of(K, rows, N)
    return {"value": adds / dt / 1e9, "unit": UNIT, "cores": nthreads, "kind": "port",
            "sample": "first %d of %d weight rows x all %d tokens x K=%d (%d LNS adds, %.1f s)" % (rows, M, N, K, adds, dt)}


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    nthreads = os.cpu_count() or 1
    vals = []
    for _ in range(args.warmup):
        cpu_leg(wl, args.mode, 0.5, nthreads)
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
        "config": {"workload": wl["desc"] + " [bounded sample per step on host cores]", "mode": args.mode},
        "cpu_baseline": leg, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


# ------------------------------------------------------------------ GPU

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

    K, M, N = wl["K"], wl["M"], wl["N"]
    strong = wl.get("strong", False)
    if strong:
        from lnsb200 import shard
        if M % world:
            raise SystemExit("configs4 needs the 8192 rows to divide by the GPU count")
        M = M // world                       # this rank's rows
    ks = lnsb200.KernelSet(16, args.mode)
    ks.upload_tables()
    rng = np.random.default_rng(wl["seed"] + 1000 * rank)
    w_f32 = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32)).cuda()    # ggml src0 rows
    x_f32 = torch.from_numpy(rng.normal(0, 1, (N, K)).astype(np.float32)).cuda()
    w = torch.empty(K * M, dtype=torch.int16, device="cuda")                          # k-major codes
    x = torch.empty(N * K, dtype=torch.int16, device="cuda")
    ks.to_lns_transposed(w_f32, w, M, K, M)
    ks.to_lns(x_f32, x)
    out = torch.empty(N * M, dtype=torch.int16, device="cuda")
    from lnsb200 import shard
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.int32, device="cuda")          # 256 MB > L2 (126 MB)
    stream = torch.cuda.current_stream()

    # the timed call goes straight to the C ABI with prebuilt arguments, so
    # host-side Python work cannot open gaps inside the event-timed region
    lib = ks.lib
    mm_args = lnsb200.MulMatArgs(w.data_ptr(), x.data_ptr(), None, K, M, N, 1, 1, 1, 1, 7)
    mm_argp = ctypes.byref(mm_args)
    out_p = ctypes.c_void_p(out.data_ptr())
    stream_p = ctypes.c_void_p(stream.cuda_stream)
    mm = lib.lnsb_mul_mat_lns
    status = [0]

    # N > 1, weak scaling: the all-gather of the output-row shards fused into
    # the mul_mat's store over NVLink peer memory (a symmetric-memory buffer
    # on every GPU, plain stores), then a device-side barrier; NCCL's
    # all-gather where the fused store does not apply
    gather = "nccl all_gather_into_tensor + permute"
    peer = None
    if world > 1 and not strong and args.mode in ("base", "monte"):
        try:
            import torch.distributed._symmetric_memory as symm_mem
            gbuf = symm_mem.empty(N * M * world, dtype=torch.int16, device="cuda")
            hdl = symm_mem.rendezvous(gbuf, dist.group.WORLD)
            fbuf = symm_mem.empty(world, dtype=torch.int32, device="cuda")
            fbuf.zero_()
            fhdl = symm_mem.rendezvous(fbuf, dist.group.WORLD)
            berr = torch.zeros(1, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            dist.barrier()
            peer = lnsb200._lib.PeerOut(hdl.buffer_ptrs_dev, world, M * world, rank * M)
            peer_p = ctypes.byref(peer)
            mmp = lib.lnsb_mul_mat_lns_peers
            epoch = [0]
            gather = "fused into the mul_mat store: peer-memory stores over NVLink + a bounded peer-flag barrier"
        except Exception as e:                                     # noqa: BLE001
            peer = None
            gather = "nccl all_gather_into_tensor + permute (symmetric memory unavailable: %s)" % str(e).splitlines()[0][:120]

    def launch():
        st = mmp(16, mm_argp, peer_p, stream_p) if peer is not None else mm(16, mm_argp, out_p, stream_p)
        if st != 0:
            status[0] = st

    def gather_step():
        if peer is not None:
            epoch[0] += 1
            st = lib.lnsb_group_barrier(ctypes.c_void_p(fhdl.buffer_ptrs_dev), world, rank, epoch[0],
                                        ctypes.c_void_p(berr.data_ptr()), stream_p)
            if st != 0:
                status[0] = st
        else:
            shard.all_gather_rows(out.view(N, M), world).contiguous()

    def step():
        launch()
        if world > 1:
            gather_step()

    if peer is not None:
        # the fused gather must give what NCCL's does, bit for bit
        gbuf.fill_(-1)
        torch.cuda.synchronize()
        dist.barrier()
        launch()
        gather_step()
        mm(16, mm_argp, out_p, stream_p)
        want = shard.all_gather_rows(out.view(N, M), world).contiguous().view(-1)
        torch.cuda.synchronize()
        if berr.item() != 0:
            raise SystemExit("peer barrier timed out")
        if not torch.equal(gbuf, want):
            raise SystemExit("fused peer all-gather differs from the NCCL all-gather")

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()

    bus = None
    try:
        p = torch.cuda.get_device_properties(local)
        bus = "%02x:%02x.0" % (p.pci_bus_id, p.pci_device_id)
    except Exception:
        pass
    sampler = ClockSampler(bus)
    sampler.start()
    time.sleep(0.4)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.zero_()                      # untimed: L2 flushed before every step
        ev[i][0].record(stream)
        launch()
        ev[i][1].record(stream)
        if world > 1:
            gather_step()                  # ggml [N][M*world] order on every GPU
        ev[i][2].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    if status[0] != 0:
        raise lnsb200.LnsbError(lib, "lnsb_mul_mat_lns", status[0])
    if peer is not None and berr.item() != 0:
        raise SystemExit("peer barrier timed out")
    step_ms = sum(a.elapsed_time(c) for a, b, c in ev)
    kern_ms = sum(a.elapsed_time(b) for a, b, c in ev)
    if dist:
        t = torch.tensor([step_ms, kern_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, kern_ms = t.tolist()

    # e2e through the C ABI with host buffers: every step uploads its F32
    # activations from pinned host memory (H2D), converts them (to_lns), runs
    # mul_mat with F32 out and reads the F32 result back into pinned host
    # memory (D2H); the weights stay resident, as the reference's weight cache
    # keeps them.  Steps are double buffered the way a serving loop runs them:
    # step i+1's upload and step i's read-back go on their own copy streams,
    # so the copies overlap the kernels of the neighbouring steps.
    NB = 2
    xh = torch.from_numpy(rng.normal(0, 1, (N, K)).astype(np.float32)).pin_memory()
    yh = [torch.empty(N * M, dtype=torch.float32).pin_memory() for _ in range(NB)]
    xd = [torch.empty(N * K, dtype=torch.float32, device="cuda") for _ in range(NB)]
    xc = [torch.empty(N * K, dtype=torch.int16, device="cuda") for _ in range(NB)]
    yd = [torch.empty(N * M, dtype=torch.float32, device="cuda") for _ in range(NB)]
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_up = [torch.cuda.Event() for _ in range(NB)]        # input b uploaded
    ev_cv = [torch.cuda.Event() for _ in range(NB)]        # input b converted: xd[b] free
    ev_mm = [torch.cuda.Event() for _ in range(NB)]        # result b computed
    ev_dn = [torch.cuda.Event() for _ in range(NB)]        # result b read back: yd[b] free

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
        ks.to_lns(xd[b], xc[b], stream=stream)
        ev_cv[b].record(stream)
        ks.mul_mat(w, xc[b], yd[b], K, M, N, monte_seed=7, stream=stream)
        ev_mm[b].record(stream)

    def download(i):
        b = i % NB
        down.wait_event(ev_mm[b])
        with torch.cuda.stream(down):
            yh[b].copy_(yd[b], non_blocking=True)
        ev_dn[b].record(down)

    def e2e_run(n):
        up.wait_stream(stream)
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)
            download(i)
        stream.wait_event(ev_dn[(n - 1) % NB])

    e2e_run(max(3, args.warmup))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
        dist.barrier()

    adds = adds_of(K, M, N)
    wkey = "configs4:%d:%d" % (K, N) if strong else args.workload
    pkey = (wkey, args.mode) if world == 1 or not strong else None   # the captured launch is this rank's launch
    value = adds * world * args.steps / (step_ms / 1000) / 1e9
    e2e_val = adds * world * args.steps / (e2e_ms / 1000) / 1e9
    scaling = "strong" if strong else "weak"
    kern_s = kern_ms / 1000 / args.steps
    hbm, smmax, src = peaks()
    f_mhz = clocks.get("sm_mhz") or smmax
    c = C_MODE.get(args.mode, 18)
    int_peak = SMS * LANES_PER_SM * f_mhz * 1e6 / c / 1e9
    achieved = adds / kern_s / 1e9
    bytes_alg = algorithmic_bytes(K, M, N)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_ms / args.steps, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": "u16 (xlns16 codes; integer LNS arithmetic)", "data": "synthetic",
        "config": {"workload": wl["desc"] + ((" per rank" if not strong else "") + ", output rows sharded + all-gather (config.gather)" if world > 1 else ""),
                   "K": K, "M": M, "N": N, "mode": args.mode, "parallelism": "rowshard%d" % world, "gather": gather if world > 1 else None,
                   "l2": "flushed (256 MB write) before every timed step"},
        "roofline": {"bound": "int", "achieved": achieved, "peak": int_peak, "unit": UNIT, "frac": achieved / int_peak,
                     "traffic": traffic_of(pkey), "traffic_source": PROFILE.get(pkey),
                     "c_mode": c, "sm_mhz_used": f_mhz,
                     "note": "integer-issue bound: %d SMs x %d lanes x f_sm / c_mode (%s SM clock)" % (SMS, LANES_PER_SM, "sampled" if clocks.get("sm_mhz") else src),
                     "hbm": {"achieved_gbs": bytes_alg / kern_s / 1e9, "peak_gbs": hbm, "frac": bytes_alg / kern_s / 1e9 / hbm,
                             "algorithmic_bytes": bytes_alg}},
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": N * K * 4, "d2h_bytes_per_step": N * M * 4,
                "path": "per step: H2D of F32 activations (pinned), lnsb_to_lns, lnsb_mul_mat (F32 out), D2H of the F32 "
                        "result (pinned); double buffered, copies on their own streams overlapping neighbouring steps"},
        "gpu_launches": args.steps * (2 if peer is not None else 1),   # mul_mat (+ the peer barrier)
        "clocks": clocks,
    }
    if world == 1 and args.workload == "configs1":
        # BASELINE's metric is quoted at K=1536: configs[0], timed the same way, beside the main line
        line["k1536"] = time_secondary(lib, lnsb200, torch, np, WORKLOADS["configs0"], args, flush, stream)
        # the rows beside the path: MUL_MAT_ID and the typed weight decode
        line["mul_mat_id"] = time_mul_mat_id(lnsb200, torch, np, args, flush, stream, int_peak)
        line["weights"] = time_weights(lnsb200, torch, np, args, flush, stream, hbm)
        line["normalisers"] = time_norms(lnsb200, torch, np, args, flush, stream)
    if args.workload == "configs1" and not args.no_decode:
        # the metric's second half: model decode tok/s, one sequence per GPU
        line["decode"] = run_decode(torch, dist, rank, world, args, cpu=(rank == 0 and world == 1 and not args.no_cpu_baseline))
        if world == 1:
            # the same model and prompt in LNS32, on 1 GPU
            line["decode_lns32"] = run_decode(torch, dist, rank, world, args,
                                              cpu=(rank == 0 and not args.no_cpu_baseline), fmt=32)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not strong:
        line["cpu_baseline"] = cpu_leg(wl, args.mode, 10.0, os.cpu_count() or 1)
        # the reference's CPU backend runs one thread (its ops are sequential loops): the
        # same port on one core, beside the all-cores figure
        line["cpu_baseline"]["single_thread"] = cpu_leg(wl, args.mode, 5.0, 1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def time_secondary(lib, lnsb200, torch, np, wl, args, flush, stream):
    """Device-timed steps of another workload through the same C ABI call (inputs
    resident, L2 flushed before every step), for a sub-object of the JSON line."""
    K, M, N = wl["K"], wl["M"], wl["N"]
    ks = lnsb200.KernelSet(16, args.mode)
    rng = np.random.default_rng(wl["seed"])
    w_f32 = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32)).cuda()
    x_f32 = torch.from_numpy(rng.normal(0, 1, (N, K)).astype(np.float32)).cuda()
    w = torch.empty(K * M, dtype=torch.int16, device="cuda")
    x = torch.empty(N * K, dtype=torch.int16, device="cuda")
    ks.to_lns_transposed(w_f32, w, M, K, M)
    ks.to_lns(x_f32, x)
    out = torch.empty(N * M, dtype=torch.int16, device="cuda")
    a = lnsb200.MulMatArgs(w.data_ptr(), x.data_ptr(), None, K, M, N, 1, 1, 1, 1, 7)
    ap, op, sp = ctypes.byref(a), ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream.cuda_stream)
    for _ in range(args.warmup):
        flush.zero_()
        if lib.lnsb_mul_mat_lns(16, ap, op, sp) != 0:
            raise RuntimeError("lnsb_mul_mat_lns failed on the K=1536 workload")
    torch.cuda.synchronize()
    steps = max(args.steps, 20)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        ev[i][0].record(stream)
        lib.lnsb_mul_mat_lns(16, ap, op, sp)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    ms = sum(b.elapsed_time(e) for b, e in ev) / steps
    adds = adds_of(K, M, N)
    return {"workload": wl["desc"], "mode": args.mode, "steps": steps, "ms_per_step": ms,
            "value": adds / (ms / 1000) / 1e9, "unit": UNIT,
            "bound": "chain latency: %d dependent additions per output" % (K - 1),
            "l2": "flushed (256 MB write) before every timed step"}


def time_norms(lnsb200, torch, np, args, flush, stream):
    """BASELINE configs[1]'s normalisers on xlns16 codes, device-timed, L2
    flushed before every step: soft_max over logits N(0, 3) shaped [9 heads]
    [512 queries][512 keys] with a causal mask (keys after the query are
    -inf) and scale 1.0 (4,608 rows x 511 additions, masked zeros included),
    and rms_norm over 512 rows of 576 N(0, 1) values, eps 1e-5 (576 additions
    per row); inputs numpy default_rng(1), converted to codes on the device."""
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
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())                        # noqa: E731
    calls = {
        "soft_max": (lambda: lib.lnsb_soft_max_lns(16, P(sm_src), ne, P(mask), mne, 0x4000, P(sm_dst), P(sm_work), 7, sp),
                     h * q * (n - 1), "chain latency: %d dependent additions per row, %d rows" % (n - 1, h * q),
                     "[9][512][512] xlns16 logits N(0,3), causal mask, scale 1.0"),
        "rms_norm": (lambda: lib.lnsb_rms_norm_lns(16, P(rn_src), P(rn_dst), cols, rows, ctypes.c_float(1e-5), 7, sp),
                     rows * cols, "chain latency: %d dependent additions per row, %d rows" % (cols, rows),
                     "512 x 576 xlns16 values N(0,1), eps 1e-5"),
    }
    out = {}
    steps = max(args.steps, 20)
    for name, (call, adds, bound, what) in calls.items():
        for _ in range(args.warmup):
            flush.zero_()
            if call() != 0:
                raise RuntimeError("lnsb_%s_lns failed" % name)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.zero_()
            ev[i][0].record(stream)
            call()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        ms = sum(b.elapsed_time(e) for b, e in ev) / steps
        out[name] = {"workload": "BASELINE configs[1] %s: %s" % (name, what), "mode": args.mode, "steps": steps,
                     "ms_per_step": ms, "value": adds / (ms / 1000) / 1e9, "unit": UNIT, "adds": adds, "bound": bound,
                     "l2": "flushed (256 MB write) before every timed step"}
    return out


def time_mul_mat_id(lnsb200, torch, np, args, flush, stream, int_peak):
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
    for _ in range(max(3, args.warmup)):
        ks.mul_mat_id_lns(w, x, ids, out, K, M, n_exp, 1, n_used, n_tok, stream=stream)
    torch.cuda.synchronize()
    steps = max(args.steps, 10)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        ev[i][0].record(stream)
        ks.mul_mat_id_lns(w, x, ids, out, K, M, n_exp, 1, n_used, n_tok, stream=stream)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    ms = sum(b.elapsed_time(e) for b, e in ev) / steps
    adds = n_tok * n_used * M * (K - 1)
    val = adds / (ms / 1000) / 1e9
    return {"workload": "MUL_MAT_ID: 8 experts of 1536x576, 128 tokens x 2 experts (synthetic, seed 4)",
            "mode": args.mode, "steps": steps, "ms_per_step": ms, "value": val, "unit": UNIT,
            "roofline": {"bound": "int", "achieved": val, "peak": int_peak, "frac": val / int_peak, "unit": UNIT},
            "l2": "flushed (256 MB write) before every timed step"}


def time_weights(lnsb200, torch, np, args, flush, stream, hbm):
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
        for _ in range(3):
            ks.to_lns_transposed_typed(t, raw, dst, rows, cols, rows, stream=stream)
        torch.cuda.synchronize()
        n = 10
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i in range(n):
            flush.zero_()
            ev[i][0].record(stream)
            ks.to_lns_transposed_typed(t, raw, dst, rows, cols, rows, stream=stream)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        ms = sum(b.elapsed_time(e) for b, e in ev) / n
        by = rows * rb + rows * cols * 2
        out[t] = {"ms": ms, "gbs": by / (ms / 1000) / 1e9, "frac_hbm": by / (ms / 1000) / 1e9 / hbm,
                  "bytes": by}
    return {"workload": "8192 x 4096 weight -> xlns16 k-major image, per storage type", "bound": "hbm",
            "peak_gbs": hbm, "types": out,
            "l2": "flushed (256 MB write) before every timed launch", "launches_per_type": 10}


def run_decode(torch, dist, rank, world, args, cpu=False, fmt=16):
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
    dec.prepare(len(prompt), len(prompt) + 127)          # captured once before the timed region
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e[0].record(stream)
    logits = model.forward(g, cfg, prompt, 0)
    toks = [g.argmax(logits)]
    e[1].record(stream)
    toks += dec.decode(toks[0], len(prompt), 127)       # each step's token copied to pinned host memory
    e[2].record(stream)
    torch.cuda.synchronize()
    pre_ms, dec_ms = e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])
    if dist:
        t = torch.tensor([pre_ms, dec_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre_ms, dec_ms = t.tolist()
    out = {"model": "SmolLM2-135M shape (30 layers, d 576, 9/3 heads, ffn 1536, vocab 49152), random N(0,0.02) weights seed 2",
           "format": "xlns%d" % fmt, "mode": args.decode_mode if fmt == 16 else None, "prompt": 128, "generated": 128, "sequences": world,
           "prefill_tok_per_s": world * 128 / (pre_ms / 1000), "decode_tok_per_s": world * 127 / (dec_ms / 1000),
           "ms_per_token": dec_ms / 127, "prefill_ms": pre_ms,
           "timing": "device events; prefill eager, decode as one CUDA graph per position (captured before the timed region); each step's greedy token is copied to pinned host memory",
           "first_tokens": toks[:8]}
    if cpu:
        # the CPU oracle (the reference's algorithm, host cores) on a bounded sample:
        # prefill of 8 tokens, then 16 decode steps (a few seconds)
        import time
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        o = model.OracleOps(cfg, w, mode=args.decode_mode, n_ctx=32, nthreads=os.cpu_count() or 1, fmt=fmt)
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
    if args.workload == "configs4":
        # 8192 x K weights, K x N activations, seed 3; output rows
        # sharded across the ranks (strong scaling), gathered with NCCL
        wl = dict(desc="BASELINE configs[4] LNS16 mul_mat sweep: W 8192x%d x X %dx%d, rows sharded"
                       % (args.sweep_k, args.sweep_k, args.sweep_n),
                  K=args.sweep_k, M=8192, N=args.sweep_n, seed=3, strong=True)
    else:
        wl = WORKLOADS[args.workload]
    if args.mode is None:
        args.mode = "sum32" if args.workload == "configs4" else "base"
    if args.impl == "reference":
        return run_reference(args, wl)
    return run_ours(args, wl)


if __name__ == "__main__":
    sys.exit(main())
