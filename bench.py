"""Benchmark of the paged-GQA decode on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1..c5] [--kv bf16|fp8] [--no-e2e] [--no-cpu-baseline]

A step is one decode call over one batch of the workload.  Workload: config c2 (long
context, B=2, Hq=64, Hkv=8, L=32768) at N=1; at N>1 (torchrun, one rank per GPU) config c5
(B=512, Hq=64, Hkv=8, L=16384, ~34 GB of KV) split by KV head, each rank owning Hkv/N heads
and their pool (strong scaling, no collective in the timed region).  `--config` overrides.

value      aggregate algorithmic KV GB/s = sum over ranks of KV bytes per call x K /
           max-over-ranks device time (CUDA events, barrier + synchronize around K steps),
           inputs resident in HBM; input copies rotate so the read set is > 4x L2.
e2e        the same metric through the reference's C symbol `run_kernel` with pinned host
           buffers: every step copies the inputs host->device, runs the decode and reads the
           output back.
roofline   achieved = algorithmic bytes per launch / mean launch time, against the measured
           HBM copy bandwidth in MEASURED_PEAKS.json; traffic from the committed ncu summary.
cpu_baseline  the CPU oracle (fp32 PyTorch paged attention, all host threads) on a bounded
           sample of the same workload, rank 0 at N=1 only.

scaling_reference  (N=1 lines) c5, the workload the N>1 runs shard, on this one GPU.

--seqlen-q S decodes S query tokens per sequence with the end-aligned causal mask
(speculative / multi-token decode, an extension): value still counts the KV bytes once.

--kv fp8 runs the same workload with e4m3 KV pages (per-KV-head scales; an extension,
the reference's pools are bf16): value counts the e4m3 bytes; no e2e or CPU leg.

--impl reference times that CPU implementation alone (the reference's path has no GPU
implementation that runs on this machine).
"""
import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

L2_BYTES = 126 * 1024 * 1024
DEFAULT_PEAK_GBS = 6650.0  # fallback when MEASURED_PEAKS.json is absent
METRIC = "KV-cache HBM GB/s (% of B200 peak) and us per paged-GQA decode call"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=None, choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-scaling-ref", action="store_true",
                    help="skip the single-GPU c5 measurement added to N=1 lines")
    ap.add_argument("--e2e-host-budget-gb", type=float, default=8.0)
    ap.add_argument("--out", default=None, help="also append the JSON line to this file")
    ap.add_argument("--profile", type=int, default=0,
                    help="run N decode calls of the workload and exit (for ncu captures)")
    ap.add_argument("--seqlen-q", type=int, default=1,
                    help="query tokens per sequence (causal, end-aligned; >1 is speculative / "
                         "multi-token decode, an extension of the reference)")
    ap.add_argument("--kv", default="bf16", choices=["bf16", "fp8"],
                    help="KV page format: bf16 (the reference's) or e4m3 with per-head scales")
    return ap.parse_args()


def measured_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return DEFAULT_PEAK_GBS, "fallback"


def committed_traffic(workload):
    """dram read+write bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None
        self.marks = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append((time.time(), parts))

    def mark(self, tag):
        self.marks.append((tag, time.time()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0, t1):
        rows = [p for (t, p) in self.samples if t0 <= t <= t1] or [p for _, p in self.samples]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[0]) for r in rows if num(r[0]) is not None]
        mx = [num(r[1]) for r in rows if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def workload_for(args, world):
    if args.config:
        return args.config
    return "c2" if world == 1 else "c5"


def describe(name, world):
    from mx_flash_attn_kernel_opt__b200 import inputs
    cfg = inputs.CONFIGS[name]
    return (f"{name}: B={cfg['B']} Hq={cfg['Hq']} Hkv={cfg['Hkv']} D=128 P={cfg['P']}; "
            f"{cfg['desc']}" + (f"; KV heads sharded over {world} GPUs" if world > 1 else ""))


# --------------------------------------------------------------------------------------
# CPU side (oracle): the cpu_baseline leg and the reference arm
# --------------------------------------------------------------------------------------

def cpu_sample_inputs(name, kv_range=None):
    """Bounded CPU sample of workload `name`: whole workload when it is small, else the
    first sequences (same lengths / layout)."""
    from mx_flash_attn_kernel_opt__b200 import inputs
    limit = {"c1": None, "c2": None, "c3": 64, "c4": 16, "c5": 2}[name]
    return inputs.baseline_config(name, batch_limit=limit, kv_head_range=kv_range), limit


def time_cpu_oracle(name, budget_s=10.0, min_calls=1, max_calls=None):
    import torch
    from oracle import paged_decode_ref
    torch.set_num_threads(os.cpu_count() or 1)
    inp, limit = cpu_sample_inputs(name)
    paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, inp.scale)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, inp.scale)
        n += 1
        el = time.perf_counter() - t0
        if (n >= min_calls and el >= budget_s) or (max_calls and n >= max_calls):
            break
    per_call = el / n
    sample = (f"{'all' if limit is None else 'first %d' % limit} of {inp.batch} sequences "
              f"of {name}, {n} calls, {inp.kv_bytes() / 1e6:.1f} MB KV per call")
    return {"value": inp.kv_bytes() / per_call / 1e9, "unit": "GB/s",
            "us_per_call": per_call * 1e6, "cores": torch.get_num_threads(), "kind": "port",
            "sample": sample}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return None
    name = workload_for(args, world)
    steps = args.steps if args.steps is not None else 3
    warm = args.warmup if args.warmup is not None else 1
    import torch
    from oracle import paged_decode_ref
    torch.set_num_threads(os.cpu_count() or 1)
    inp, limit = cpu_sample_inputs(name)
    for _ in range(warm):
        paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, inp.scale)
    t0 = time.perf_counter()
    for _ in range(steps):
        paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, inp.scale)
    el = time.perf_counter() - t0
    per = el / steps
    gbs = inp.kv_bytes() / per / 1e9
    sample = (f"{'all' if limit is None else 'first %d' % limit} of the sequences of {name}; "
              f"{inp.kv_bytes() / 1e6:.1f} MB KV per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": per * 1e3,
        "us_per_call": per * 1e6, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": describe(name, 1), "sample": sample},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s",
                         "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": ("the reference's implementations need MetaX mxcc (C++) or run only as an "
                 "fp32 restatement on the host; timed: oracle/paged_decode.py "
                 "(fp32 PyTorch paged attention), all host threads"),
    }
    return line


# --------------------------------------------------------------------------------------
# GPU side
# --------------------------------------------------------------------------------------

def main():
    args = parse()
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.profile:
        profile_calls(args, world)
        return

    if args.impl == "reference":
        if world > 1:
            import datetime
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        line = run_reference_arm(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    from mx_flash_attn_kernel_opt__b200 import _lib, inputs, ops, sharding
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    name = workload_for(args, world)
    cfg = inputs.CONFIGS[name]
    lo, hi = sharding.kv_head_range(rank, world, cfg["Hkv"]) if world > 1 else (0, cfg["Hkv"])
    inp = inputs.baseline_config(name, device=dev, kv_head_range=(lo, hi))
    fp8 = args.kv == "fp8"
    if fp8:
        inp = inputs.to_fp8(inp, keep_device=True)
        torch.cuda.empty_cache()
    Sq = max(1, args.seqlen_q)
    if Sq > 1:  # Sq query tokens per sequence, q / out [B, Sq, Hq, D]
        g_q = torch.Generator(device=dev).manual_seed(1234)
        qm = torch.randn((inp.batch, Sq, inp.num_heads, 128), generator=g_q, device=dev)
        inp.q = qm.to(torch.bfloat16)
    kv_bytes = inp.kv_bytes()
    alg_bytes = inp.algorithmic_bytes()

    # rotate input copies so the set read between two reuses is > 4x L2
    copies = max(1, math.ceil(4 * L2_BYTES / max(kv_bytes, 1)))
    free = torch.cuda.mem_get_info(dev)[0]
    copies = max(1, min(copies, int(0.6 * free // max(2 * inp.k.numel() * inp.k.element_size(), 1)) + 1, 64))
    sets = [(inp.k, inp.v)]
    for _ in range(copies - 1):
        sets.append((inp.k.clone(), inp.v.clone()))
    out = torch.empty_like(inp.q)
    ws = ops.workspace_for(inp.batch, inp.num_heads, inp.num_heads_k, 128, inp.page_size, dev,
                           seqlen_q=Sq)
    stream = torch.cuda.current_stream(dev)

    # one correctness-checked call through the Python wrapper, then prebuilt C calls
    ops.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale, out=out,
               workspace=ws, k_scale=inp.k_scale, v_scale=inp.v_scale, causal=Sq > 1)
    L = _lib.lib()
    vp = ctypes.c_void_p
    sh = vp(stream.cuda_stream)
    if fp8:
        argsets = [(vp(inp.q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), None, None,
                    vp(out.data_ptr()), vp(inp.seq_lens.data_ptr()),
                    vp(inp.block_table.data_ptr()), inp.batch, Sq, 0, inp.num_heads,
                    inp.num_heads_k, 128, inp.page_size, inp.num_pages,
                    inp.block_table.stride(0), 0, int(Sq > 1), ctypes.c_float(inp.scale),
                    vp(inp.k_scale.data_ptr()), vp(inp.v_scale.data_ptr()), vp(ws.data_ptr()),
                    ws.numel(), sh) for (k, v) in sets]
        fn, fn_name = L.pgqa_decode_fp8, "pgqa_decode_fp8"
    elif Sq > 1:
        argsets = [(vp(inp.q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(out.data_ptr()),
                    vp(inp.seq_lens.data_ptr()), vp(inp.block_table.data_ptr()), inp.batch, Sq,
                    inp.num_heads, inp.num_heads_k, 128, inp.page_size, inp.num_pages,
                    inp.block_table.stride(0), 0, 1, ctypes.c_float(inp.scale), vp(ws.data_ptr()),
                    ws.numel(), sh) for (k, v) in sets]
        fn, fn_name = L.pgqa_decode_v2, "pgqa_decode_v2"
    else:
        argsets = [(vp(inp.q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(out.data_ptr()),
                    vp(inp.seq_lens.data_ptr()), vp(inp.block_table.data_ptr()), inp.batch,
                    inp.num_heads, inp.num_heads_k, 128, inp.page_size, inp.num_pages,
                    inp.block_table.stride(0), 0, ctypes.c_float(inp.scale), vp(ws.data_ptr()),
                    ws.numel(), sh) for (k, v) in sets]
        fn, fn_name = L.pgqa_decode_v1, "pgqa_decode_v1"

    def step(i):
        st = fn(*argsets[i % len(argsets)])
        if st != 0:
            raise _lib.PgqaError(st, fn_name)

    # warm-up: at least W steps and ~0.5 s (clock ramp-up, nvidia-smi samples)
    t_one = None
    warm = args.warmup if args.warmup is not None else 10
    warm = max(3, warm)
    phys = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    if vis:
        ids = [x.strip() for x in vis.split(",")]
        if local < len(ids) and ids[local].isdigit():
            phys = int(ids[local])
    sampler = ClockSampler(phys)
    sampler.start()
    t_w0 = time.time()
    for i in range(warm):
        step(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    step(0)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_one = max(e0.elapsed_time(e1) / 1e3, 1e-6)
    extra = 0
    while time.time() - t_w0 < 0.5 and extra < 100000:
        for i in range(max(1, int(0.05 / t_one))):
            step(i)
            extra += 1
        torch.cuda.synchronize(dev)

    steps = args.steps if args.steps is not None else max(20, min(20000, int(1.0 / t_one)))
    ops.check_device_error(ws, dev)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.mark("t0")
    t_wall0 = time.time()
    e0.record(stream)
    for i in range(steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_wall1 = time.time()
    if world > 1:
        dist.barrier()
    el_ms = e0.elapsed_time(e1)
    # keep sampling a little so a short timed region still gets clock samples
    if t_wall1 - t_wall0 < 0.45:
        tail_end = time.time() + 0.45
        while time.time() < tail_end:
            for i in range(max(1, int(0.05 / t_one))):
                step(i)
            torch.cuda.synchronize(dev)
    clocks = sampler.summary(t_wall0 - 0.25, max(t_wall1, time.time()))
    sampler.stop()
    ops.check_device_error(ws, dev)

    if world > 1:
        t = torch.tensor([el_ms, float(kv_bytes), float(alg_bytes)], dtype=torch.float64,
                         device=dev)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        el_ms_max = float(tmax[0])
        kv_total = float(tsum[1])
        alg_total = float(tsum[2])
    else:
        el_ms_max, kv_total, alg_total = el_ms, float(kv_bytes), float(alg_bytes)

    per_call_s = el_ms_max / 1e3 / steps
    value = kv_total / per_call_s / 1e9
    peak, peak_kind = measured_peak()
    # per-GPU roofline of the decode kernel on this rank (one launch per step)
    achieved = alg_bytes / (el_ms / 1e3 / steps) / 1e9

    # ---- optional all-gather of the per-rank outputs, timed separately ----
    allgather = None
    if world > 1:
        for _ in range(3):
            sharding.gather_heads(out)
        torch.cuda.synchronize(dev)
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        n_ag = 20
        for _ in range(n_ag):
            full = sharding.gather_heads(out)
        a1.record(stream)
        torch.cuda.synchronize(dev)
        ag = torch.tensor([a0.elapsed_time(a1) / n_ag], dtype=torch.float64, device=dev)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        allgather = {"us_per_call": float(ag) * 1e3,
                     "bytes_per_rank": int(out.numel() * 2 * world),
                     "shape": list(full.shape)}

    # ---- end to end through the C symbol with host buffers ----
    e2e = None
    if not args.no_e2e and not fp8 and Sq == 1:
        e2e = e2e_measure(inp, dev, stream, steps, args.e2e_host_budget_gb, world)
        if world > 1:
            t = torch.tensor([e2e.pop("_ms"), e2e.pop("_kv")], dtype=torch.float64, device=dev)
            tm = t.clone()
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            ts = t.clone()
            dist.all_reduce(ts, op=dist.ReduceOp.SUM)
            e2e["value"] = round(float(ts[1]) / (float(tm[0]) / 1e3) / 1e9, 3)
        else:
            ms, kvb = e2e.pop("_ms"), e2e.pop("_kv")
            e2e["value"] = round(kvb / (ms / 1e3) / 1e9, 3)

    scaling_ref = None
    if world == 1 and not args.no_scaling_ref and not fp8 and Sq == 1 and name != "c5":
        scaling_ref = scaling_reference(dev, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not fp8 and Sq == 1:
        cpu = time_cpu_oracle(name, budget_s=10.0)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": el_ms_max / steps,
            "us_per_call": per_call_s * 1e6, "pct_of_peak": round(100 * value / world / peak, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "e4m3 KV pages (per-KV-head fp32 scales), bf16 q/out, f16 MMA, fp32 softmax" if fp8 else "bf16",
            "data": "synthetic",
            "config": {"workload": describe(name, world),
                       "kv_bytes_per_call": int(kv_total),
                       "kv_format": args.kv,
                       "seqlen_q": Sq, "causal": Sq > 1,
                       "l2": (f"{len(sets)} rotating K/V pool copies, "
                              f"{len(sets) * kv_bytes / 1e6:.0f} MB read set per rank "
                              f"(> L2 {L2_BYTES / 1e6:.0f} MB)"),
                       "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                         "bytes_per_launch": int(alg_bytes),
                         "traffic": committed_traffic((name if world == 1 else f"{name}/x{world}")
                                                      + ("/fp8" if fp8 else "")),
                         "kernel": "pgqa_decode_kernel"},
            "gpu_launches": steps,
            "clocks": clocks,
            "e2e": e2e,
            "impl": "ours",
        }
        if allgather is not None:
            line["allgather"] = allgather
        if scaling_ref is not None:
            line["scaling_reference"] = scaling_ref
        if cpu is not None:
            line["cpu_baseline"] = cpu
        s = json.dumps(line)
        print(s, flush=True)
        if args.out:
            with open(args.out, "a") as f:
                f.write(s + "\n")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def profile_calls(args, world):
    """N back-to-back decode calls of the workload on cuda:0, no timing (ncu driver)."""
    import torch
    from mx_flash_attn_kernel_opt__b200 import inputs, ops
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    name = workload_for(args, world)
    inp = inputs.baseline_config(name, device=dev)
    if args.kv == "fp8":
        inp = inputs.to_fp8(inp, keep_device=True)
    out = torch.empty_like(inp.q)
    ws = ops.workspace_for(inp.batch, inp.num_heads, inp.num_heads_k, 128, inp.page_size, dev)
    for _ in range(args.profile):
        ops.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale, out=out,
                   workspace=ws, k_scale=inp.k_scale, v_scale=inp.v_scale)
    torch.cuda.synchronize(dev)
    ops.check_device_error(ws, dev)
    print(json.dumps({"profile_calls": args.profile, "workload": name, "kv": args.kv}))


def scaling_reference(dev, stream, steps=10):
    """The multi-GPU workload (c5, all KV heads) on this one GPU: the N=1 point of the
    scaling series that bench.py runs at N>1 (device time, same method as `value`)."""
    import torch
    from mx_flash_attn_kernel_opt__b200 import _lib, inputs, ops
    inp = inputs.baseline_config("c5", device=dev)
    out = torch.empty_like(inp.q)
    ws = ops.workspace_for(inp.batch, inp.num_heads, inp.num_heads_k, 128, inp.page_size, dev)
    vp = ctypes.c_void_p
    args = (vp(inp.q.data_ptr()), vp(inp.k.data_ptr()), vp(inp.v.data_ptr()), vp(out.data_ptr()),
            vp(inp.seq_lens.data_ptr()), vp(inp.block_table.data_ptr()), inp.batch,
            inp.num_heads, inp.num_heads_k, 128, inp.page_size, inp.num_pages,
            inp.block_table.stride(0), 0, ctypes.c_float(inp.scale), vp(ws.data_ptr()),
            ws.numel(), vp(stream.cuda_stream))
    L = _lib.lib()
    for _ in range(3):
        _lib.check(L.pgqa_decode_v1(*args), "pgqa_decode_v1")
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        L.pgqa_decode_v1(*args)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ops.check_device_error(ws, dev)
    per = e0.elapsed_time(e1) / 1e3 / steps
    kvb = inp.kv_bytes()
    del inp, out
    torch.cuda.empty_cache()
    return {"workload": describe("c5", 1), "n_gpus": 1, "steps": steps,
            "us_per_call": round(per * 1e6, 2), "value": round(kvb / per / 1e9, 3), "unit": "GB/s",
            "note": "bench.py at N>1 runs this workload sharded by KV head; read scaling "
                    "against this value (the N=1 line's `value` is the c2 headline)"}


def e2e_measure(inp, dev, stream, steps, budget_gb, world):
    """Decode through the C `run_kernel` with host buffers: per step H2D of q, K, V,
    block table and lengths from pinned memory, the call, D2H of the output."""
    import torch
    from mx_flash_attn_kernel_opt__b200 import ops
    B = inp.batch
    per_seq = (inp.k.numel() * 2 * 2) / B
    limit = B
    if inp.k.numel() * 4 > budget_gb * 1e9:
        # host sample: the first sequences and their pages only
        limit = max(1, int(budget_gb * 1e9 // max(per_seq, 1)))
    if limit < B:
        P = inp.page_size
        seqs = inp.seq_lens[:limit].cpu()
        npg = ((seqs + P - 1) // P).tolist()
        bt_rows = inp.block_table[:limit].cpu()
        ids = torch.cat([bt_rows[b, :npg[b]] for b in range(limit)]).to(torch.int64)
        width = max(npg)
        k_h = inp.k.index_select(0, ids.to(dev)).cpu()
        v_h = inp.v.index_select(0, ids.to(dev)).cpu()
        bt = torch.zeros(limit, width, dtype=torch.int32)
        pos = 0
        for b in range(limit):
            bt[b, :npg[b]] = torch.arange(pos, pos + npg[b], dtype=torch.int32)
            pos += npg[b]
        q_h, sl_h = inp.q[:limit].cpu(), seqs
        note = f"first {limit} of {B} sequences (host budget {budget_gb} GB)"
    else:
        q_h, k_h, v_h = inp.q.cpu(), inp.k.cpu(), inp.v.cpu()
        bt, sl_h = inp.block_table.cpu(), inp.seq_lens.cpu()
        note = "whole workload"
    # the reference ABI needs pool = batch * row width
    nb = k_h.shape[0]
    Bh = q_h.shape[0]
    width = bt.shape[1]
    if nb != Bh * width:
        width = max(width, -(-nb // Bh))
        bt2 = torch.zeros(Bh, width, dtype=torch.int32)
        bt2[:, :bt.shape[1]] = bt
        bt = bt2
        pad = Bh * width - nb
        if pad:
            k_h = torch.cat([k_h, torch.zeros((pad,) + tuple(k_h.shape[1:]), dtype=k_h.dtype)])
            v_h = torch.cat([v_h, torch.zeros((pad,) + tuple(v_h.shape[1:]), dtype=v_h.dtype)])
    hq = [t.pin_memory() for t in (q_h, k_h, v_h, bt, sl_h)]
    dq = [torch.empty_like(t, device=dev) for t in hq]
    out_d = torch.empty_like(dq[0])
    out_h = torch.empty_like(hq[0]).pin_memory()
    Hq, D = q_h.shape[1], q_h.shape[2]
    Hkv, P = k_h.shape[2], k_h.shape[1]
    seqlen_k = int(sl_h.max())
    legacy = torch.cuda.default_stream(dev)
    h2d = sum(t.numel() * t.element_size() for t in hq)
    d2h = out_h.numel() * out_h.element_size()
    kvb = int(sl_h.to(torch.int64).sum()) * Hkv * D * 4

    def one():
        for d, h in zip(dq, hq):
            d.copy_(h, non_blocking=True)
        ops.run_kernel_cabi(dq[0], dq[1], dq[2], out_d, dq[4], dq[3], Bh, seqlen_k, 1, Hq, Hkv,
                            D, P, k_h.shape[0], 0)
        out_h.copy_(out_d, non_blocking=True)

    n = max(3, min(steps, 20))
    with torch.cuda.stream(legacy):
        one()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(legacy)
        for _ in range(n):
            one()
        e1.record(legacy)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / n
    return {"unit": "GB/s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "steps": n, "ms_per_step": ms, "sample": note, "path": "C run_kernel (ctypes)",
            "_ms": ms, "_kv": float(kvb)}


if __name__ == "__main__":
    main()
