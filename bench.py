"""Benchmark of the paged-GQA decode on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1..c5] [--kv bf16|fp8] [--seqlen-q S]
                    [--no-e2e] [--no-cpu-baseline] [--no-per-config]

A step is one decode call over one batch of the workload.  The headline workload is
config c5 (B=512, Hq=64, Hkv=8, L=16384, ~34 GB of KV) at every N: at N=1 on one GPU,
at N>1 (torchrun, one rank per GPU) split by KV head, each rank owning Hkv/N heads and
their pool (no collective in the timed region).  c5 is the largest named configuration
that fits one GPU and the one the multi-GPU runs shard, so per-N values divide like by
like.  `--config` overrides the workload.

value      aggregate algorithmic KV GB/s = sum over ranks of KV bytes per call x K /
           max-over-ranks device time (CUDA events, barrier + synchronize around K steps),
           inputs resident in HBM and larger than L2 (smaller workloads rotate K/V pool
           copies so that the set read between two reuses is > 4x L2).
per_config (N=1) every named configuration c1..c5 timed the same way, one after the
           other (the reference harness's per-case loop), each with its own roofline.
e2e        the same metric through the reference's C symbol `run_kernel` with pinned host
           buffers: every step copies the inputs host->device, runs the decode and reads
           the output back (bounded by the host-memory budget; the sample is named).
roofline   achieved = algorithmic bytes per launch / mean launch time, against the measured
           HBM copy bandwidth in MEASURED_PEAKS.json; traffic from the committed ncu table.
cpu_baseline  the CPU oracle (fp32 PyTorch paged attention, all host threads) on a bounded
           sample of the same workload, rank 0 at N=1 only.

--seqlen-q S decodes S query tokens per sequence with the end-aligned causal mask
(speculative / multi-token decode, an extension): value still counts the KV bytes once.
--kv fp8 runs with e4m3 KV pages (per-KV-head scales; an extension, the reference's
pools are bf16): value counts the e4m3 bytes; no e2e or CPU leg.

--impl reference times the reference's path on the host cores: the fp32 oracle (the
reference's kernels need MetaX hardware and no GPU implementation of it runs here), on
the same config, metric and unit; under torchrun only rank 0 runs it.
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
HEADLINE = "c5"
NAMED = ("c1", "c2", "c3", "c4", "c5")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=None, choices=list(NAMED))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per-configuration lines of N=1 runs")
    ap.add_argument("--e2e-host-budget-gb", type=float, default=48.0)
    ap.add_argument("--out", default=None, help="also append the JSON line to this file")
    ap.add_argument("--profile", type=int, default=0,
                    help="run N decode calls of the workload and exit (for ncu captures)")
    ap.add_argument("--batch-limit", type=int, default=None,
                    help="with --profile: keep only the first sequences of the workload "
                         "(a small capture of a workload too large for ncu)")
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


def traffic_key(name, world, kv, Sq):
    return (name + (f"/x{world}" if world > 1 else "") + ("/fp8" if kv == "fp8" else "")
            + (f"/sq{Sq}" if Sq > 1 else ""))


def committed_traffic(key):
    """dram read+write bytes per launch from the committed ncu table, if any."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(key)
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


def workload_for(args):
    return args.config or HEADLINE


def describe(name, world):
    from mx_flash_attn_kernel_opt__b200 import inputs
    cfg = inputs.CONFIGS[name]
    return (f"{name}: B={cfg['B']} Hq={cfg['Hq']} Hkv={cfg['Hkv']} D=128 P={cfg['P']}; "
            f"{cfg['desc']}" + (f"; KV heads sharded over {world} GPUs" if world > 1 else ""))


def rotation_copies(kv_bytes_rank):
    """K/V pool copies rotated so the set read between two reuses of one is > 4x L2."""
    return max(1, min(64, math.ceil(4 * L2_BYTES / max(kv_bytes_rank, 1))))


def config_dict(name, world, kv, Sq):
    """The `config` object of the JSON line; both arms print the same one."""
    from mx_flash_attn_kernel_opt__b200 import inputs
    cfg = inputs.CONFIGS[name]
    seq_lens, _ = inputs.config_seq_lens(name)
    elem = 1 if kv == "fp8" else 2
    kv_bytes = int(seq_lens.long().sum()) * cfg["Hkv"] * 128 * 2 * elem
    copies = rotation_copies(kv_bytes // world)
    return {"workload": describe(name, world),
            "kv_bytes_per_call": kv_bytes,
            "kv_format": kv,
            "seqlen_q": Sq, "causal": Sq > 1,
            "l2": ("inputs larger than L2: " if copies == 1 else
                   f"{copies} K/V pool copies rotate so each call's read set is > 4x L2: ")
                  + f"{copies * kv_bytes / world / 1e6:.0f} MB read per rank between reuses "
                    f"(L2 {L2_BYTES / 1e6:.0f} MB)",
            "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU"}


# --------------------------------------------------------------------------------------
# CPU side (oracle): the cpu_baseline leg and the reference arm
# --------------------------------------------------------------------------------------

CPU_SAMPLE_LIMIT = {"c1": None, "c2": None, "c3": 64, "c4": 16, "c5": 2}


def cpu_sample_inputs(name, kv_range=None):
    """Bounded CPU sample of workload `name`: the whole workload when it is small, else
    its first sequences (same lengths / layout)."""
    from mx_flash_attn_kernel_opt__b200 import inputs
    limit = CPU_SAMPLE_LIMIT[name]
    return inputs.baseline_config(name, batch_limit=limit, kv_head_range=kv_range), limit


def _sample_text(inp, limit, name):
    from mx_flash_attn_kernel_opt__b200 import inputs
    total = inputs.CONFIGS[name]["B"]
    return (f"{'all' if limit is None else 'first %d' % limit} of {total} sequences of "
            f"{name}, {inp.kv_bytes() / 1e6:.1f} MB KV per call")


def time_cpu_oracle(name, budget_s=10.0):
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
        if el >= budget_s:
            break
    per_call = el / n
    return {"value": round(inp.kv_bytes() / per_call / 1e9, 3), "unit": "GB/s",
            "us_per_call": per_call * 1e6, "cores": torch.get_num_threads(), "kind": "port",
            "sample": _sample_text(inp, limit, name) + f", {n} calls"}


def run_reference_arm(args, rank, world):
    """The reference's path on the host cores (rank 0 only; other ranks exit at once)."""
    if rank != 0:
        return None
    name = workload_for(args)
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
    sample = _sample_text(inp, limit, name)
    return {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": per * 1e3,
        "us_per_call": per * 1e6, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(name, world, "bf16", 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s",
                         "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": ("the reference's implementations need MetaX mxcc (C++) or run only as an "
                 "fp32 restatement on the host; timed: oracle/paged_decode.py "
                 "(fp32 PyTorch paged attention), all host threads, each step one call "
                 "over the sample named in cpu_baseline.sample"),
    }


# --------------------------------------------------------------------------------------
# GPU side
# --------------------------------------------------------------------------------------

class DecodeRun:
    """Inputs of one workload resident on this rank's GPU, with prebuilt C-ABI calls over
    rotating K/V pool copies."""

    def __init__(self, name, dev, stream, world, rank, kv, Sq):
        import torch
        from mx_flash_attn_kernel_opt__b200 import _lib, inputs, ops, sharding
        cfg = inputs.CONFIGS[name]
        lo, hi = sharding.kv_head_range(rank, world, cfg["Hkv"]) if world > 1 else (0, cfg["Hkv"])
        inp = inputs.baseline_config(name, device=dev, kv_head_range=(lo, hi))
        fp8 = kv == "fp8"
        if fp8:
            inp = inputs.to_fp8(inp, keep_device=True)
            torch.cuda.empty_cache()
        if Sq > 1:  # Sq query tokens per sequence, q / out [B, Sq, Hq, D]
            g_q = torch.Generator(device=dev).manual_seed(1234)
            inp.q = torch.randn((inp.batch, Sq, inp.num_heads, 128), generator=g_q,
                                device=dev).to(torch.bfloat16)
        self.name, self.dev, self.stream, self.inp, self.fp8, self.Sq = name, dev, stream, inp, fp8, Sq
        self.kv_bytes = inp.kv_bytes()
        self.alg_bytes = inp.algorithmic_bytes()
        copies = rotation_copies(self.kv_bytes)
        free = torch.cuda.mem_get_info(dev)[0]
        pool_bytes = 2 * inp.k.numel() * inp.k.element_size()
        copies = max(1, min(copies, int(0.6 * free // max(pool_bytes, 1)) + 1))
        self.sets = [(inp.k, inp.v)] + [(inp.k.clone(), inp.v.clone()) for _ in range(copies - 1)]
        self.out = torch.empty_like(inp.q)
        self.ws = ops.workspace_for(inp.batch, inp.num_heads, inp.num_heads_k, 128,
                                    inp.page_size, dev, seqlen_q=Sq)
        # one call through the Python wrapper (argument checks), then prebuilt C calls
        ops.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale,
                   out=self.out, workspace=self.ws, k_scale=inp.k_scale, v_scale=inp.v_scale,
                   causal=Sq > 1)
        L = _lib.lib()
        vp = ctypes.c_void_p
        sh = vp(stream.cuda_stream)
        ws = self.ws
        if fp8:
            self.argsets = [
                (vp(inp.q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), None, None,
                 vp(self.out.data_ptr()), vp(inp.seq_lens.data_ptr()),
                 vp(inp.block_table.data_ptr()), inp.batch, Sq, 0, inp.num_heads,
                 inp.num_heads_k, 128, inp.page_size, inp.num_pages, inp.block_table.stride(0),
                 0, int(Sq > 1), ctypes.c_float(inp.scale), vp(inp.k_scale.data_ptr()),
                 vp(inp.v_scale.data_ptr()), vp(ws.data_ptr()), ws.numel(), sh)
                for (k, v) in self.sets]
            self.fn, self.fn_name = L.pgqa_decode_fp8, "pgqa_decode_fp8"
        elif Sq > 1:
            self.argsets = [
                (vp(inp.q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(self.out.data_ptr()),
                 vp(inp.seq_lens.data_ptr()), vp(inp.block_table.data_ptr()), inp.batch, Sq,
                 inp.num_heads, inp.num_heads_k, 128, inp.page_size, inp.num_pages,
                 inp.block_table.stride(0), 0, 1, ctypes.c_float(inp.scale), vp(ws.data_ptr()),
                 ws.numel(), sh) for (k, v) in self.sets]
            self.fn, self.fn_name = L.pgqa_decode_v2, "pgqa_decode_v2"
        else:
            self.argsets = [
                (vp(inp.q.data_ptr()), vp(k.data_ptr()), vp(v.data_ptr()), vp(self.out.data_ptr()),
                 vp(inp.seq_lens.data_ptr()), vp(inp.block_table.data_ptr()), inp.batch,
                 inp.num_heads, inp.num_heads_k, 128, inp.page_size, inp.num_pages,
                 inp.block_table.stride(0), 0, ctypes.c_float(inp.scale), vp(ws.data_ptr()),
                 ws.numel(), sh) for (k, v) in self.sets]
            self.fn, self.fn_name = L.pgqa_decode_v1, "pgqa_decode_v1"
        self._lib = _lib

    def step(self, i):
        st = self.fn(*self.argsets[i % len(self.argsets)])
        if st != 0:
            raise self._lib.PgqaError(st, self.fn_name)

    def one_call_s(self):
        import torch
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        self.step(0)
        e1.record(self.stream)
        torch.cuda.synchronize(self.dev)
        return max(e0.elapsed_time(e1) / 1e3, 1e-6)

    def timed(self, steps, dist=None):
        """K back-to-back calls between CUDA events on the launching stream, bracketed by
        a barrier (multi-rank) and a synchronize on both sides.  Returns ms."""
        import torch
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(self.dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for i in range(steps):
            self.step(i)
        e1.record(self.stream)
        torch.cuda.synchronize(self.dev)
        if dist is not None:
            dist.barrier()
        return e0.elapsed_time(e1)

    def check(self):
        from mx_flash_attn_kernel_opt__b200 import ops
        ops.check_device_error(self.ws, self.dev)

    def release(self):
        import torch
        self.sets = self.argsets = self.out = None
        self.inp = None
        torch.cuda.empty_cache()


def measure_config(name, dev, stream, kv, Sq, peak, min_time_s=0.25):
    """One named configuration at N=1: >= 3 warm-up calls, then enough timed calls for
    about `min_time_s` (at least 20)."""
    run = DecodeRun(name, dev, stream, 1, 0, kv, Sq)
    try:
        for i in range(5):
            run.step(i)
        t_one = run.one_call_s()
        steps = max(20, min(20000, int(min_time_s / t_one)))
        ms = run.timed(steps)
        run.check()
        per = ms / 1e3 / steps
        achieved = run.alg_bytes / per / 1e9
        return {"workload": describe(name, 1), "us_per_call": round(per * 1e6, 3),
                "value": round(run.kv_bytes / per / 1e9, 3), "unit": "GB/s", "steps": steps,
                "rotating_copies": len(run.sets),
                "roofline": {"achieved": round(achieved, 1), "frac": round(achieved / peak, 4),
                             "bytes_per_launch": int(run.alg_bytes),
                             "traffic": committed_traffic(traffic_key(name, 1, kv, Sq))}}
    finally:
        run.release()


def main():
    args = parse()
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.profile:
        profile_calls(args)
        return

    if args.impl == "reference":
        line = run_reference_arm(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    from mx_flash_attn_kernel_opt__b200 import sharding
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    stream = torch.cuda.current_stream(dev)
    Sq = max(1, args.seqlen_q)
    name = workload_for(args)
    peak, peak_kind = measured_peak()

    # ---- every named configuration at N=1, before the headline's large pool ----
    per_config = None
    if world == 1 and not args.no_per_config:
        per_config = {}
        for c in NAMED:
            if c != name:
                per_config[c] = measure_config(c, dev, stream, args.kv, Sq, peak)

    # ---- the headline workload ----
    run = DecodeRun(name, dev, stream, world, rank, args.kv, Sq)
    warm = max(3, args.warmup if args.warmup is not None else 10)
    phys = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    if vis:
        ids = [x.strip() for x in vis.split(",")]
        if local < len(ids) and ids[local].isdigit():
            phys = int(ids[local])
    sampler = ClockSampler(phys)
    sampler.start()
    # warm-up: at least W steps and ~0.5 s (clock ramp-up, nvidia-smi samples)
    t_w0 = time.time()
    for i in range(warm):
        run.step(i)
    torch.cuda.synchronize(dev)
    t_one = run.one_call_s()
    extra = 0
    while time.time() - t_w0 < 0.5 and extra < 100000:
        for i in range(max(1, int(0.05 / t_one))):
            run.step(i)
            extra += 1
        torch.cuda.synchronize(dev)
    steps = args.steps if args.steps is not None else max(20, min(20000, int(1.0 / t_one)))
    run.check()
    t_wall0 = time.time()
    el_ms = run.timed(steps, dist if world > 1 else None)
    t_wall1 = time.time()
    # keep sampling a little so a short timed region still gets clock samples
    if t_wall1 - t_wall0 < 0.45:
        tail_end = time.time() + 0.45
        while time.time() < tail_end:
            for i in range(max(1, int(0.05 / t_one))):
                run.step(i)
            torch.cuda.synchronize(dev)
    clocks = sampler.summary(t_wall0 - 0.25, max(t_wall1, time.time()))
    sampler.stop()
    run.check()

    kv_bytes, alg_bytes = run.kv_bytes, run.alg_bytes
    if world > 1:
        t = torch.tensor([el_ms, float(kv_bytes), float(alg_bytes)], dtype=torch.float64,
                         device=dev)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        el_ms_max, kv_total = float(tmax[0]), float(tsum[1])
    else:
        el_ms_max, kv_total = el_ms, float(kv_bytes)
    per_call_s = el_ms_max / 1e3 / steps
    value = kv_total / per_call_s / 1e9
    # per-GPU roofline of the decode kernel on this rank (one launch per step)
    achieved = alg_bytes / (el_ms / 1e3 / steps) / 1e9

    # ---- optional all-gather of the per-rank outputs, timed separately ----
    allgather = None
    if world > 1:
        for _ in range(3):
            sharding.gather_heads(run.out)
        torch.cuda.synchronize(dev)
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        n_ag = 20
        for _ in range(n_ag):
            full = sharding.gather_heads(run.out)
        a1.record(stream)
        torch.cuda.synchronize(dev)
        ag = torch.tensor([a0.elapsed_time(a1) / n_ag], dtype=torch.float64, device=dev)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        allgather = {"us_per_call": float(ag) * 1e3,
                     "bytes_per_rank": int(run.out.numel() * 2 * world),
                     "shape": list(full.shape)}

    # ---- end to end through the C symbol with host buffers ----
    e2e = None
    if not args.no_e2e and run.fp8 is False and Sq == 1:
        e2e = e2e_measure(run, steps, args.e2e_host_budget_gb, world)
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
    run.release()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.kv == "bf16" and Sq == 1:
        cpu = time_cpu_oracle(name, budget_s=10.0)

    if rank == 0:
        fp8 = args.kv == "fp8"
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": el_ms_max / steps,
            "us_per_call": per_call_s * 1e6, "pct_of_peak": round(100 * value / world / peak, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("e4m3 KV pages (per-KV-head fp32 scales), bf16 q/out, f16 MMA, fp32 softmax"
                      if fp8 else "bf16"),
            "data": "synthetic",
            "config": config_dict(name, world, args.kv, Sq),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": f"{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                         "bytes_per_launch": int(alg_bytes),
                         "traffic": committed_traffic(traffic_key(name, world, args.kv, Sq)),
                         "kernel": "pgqa_decode_kernel"},
            "gpu_launches": steps,
            "clocks": clocks,
            "e2e": e2e,
            "impl": "ours",
        }
        if per_config is not None:
            head = {"workload": describe(name, 1), "us_per_call": round(per_call_s * 1e6, 3),
                    "value": round(value, 3), "unit": "GB/s", "steps": steps,
                    "rotating_copies": None,
                    "roofline": {k: line["roofline"][k]
                                 for k in ("achieved", "frac", "bytes_per_launch", "traffic")},
                    "note": "the headline measurement"}
            line["per_config"] = {c: (head if c == name else per_config[c]) for c in NAMED}
        if allgather is not None:
            line["allgather"] = allgather
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


def profile_calls(args):
    """N back-to-back decode calls of the workload on this rank's GPU, no timing (an ncu
    driver).  --batch-limit keeps the first sequences only (a small capture)."""
    import torch
    from mx_flash_attn_kernel_opt__b200 import inputs, ops
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    name = workload_for(args)
    inp = inputs.baseline_config(name, device=dev, batch_limit=args.batch_limit)
    if args.kv == "fp8":
        inp = inputs.to_fp8(inp, keep_device=True)
    Sq = max(1, args.seqlen_q)
    if Sq > 1:
        g_q = torch.Generator(device=dev).manual_seed(1234)
        inp.q = torch.randn((inp.batch, Sq, inp.num_heads, 128), generator=g_q,
                            device=dev).to(torch.bfloat16)
    out = torch.empty_like(inp.q)
    ws = ops.workspace_for(inp.batch, inp.num_heads, inp.num_heads_k, 128, inp.page_size, dev,
                           seqlen_q=Sq)
    for _ in range(args.profile):
        ops.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale, out=out,
                   workspace=ws, k_scale=inp.k_scale, v_scale=inp.v_scale, causal=Sq > 1)
    torch.cuda.synchronize(dev)
    ops.check_device_error(ws, dev)
    print(json.dumps({"profile_calls": args.profile, "workload": name, "kv": args.kv,
                      "seqlen_q": Sq, "batch": inp.batch,
                      "algorithmic_bytes": inp.algorithmic_bytes()}))


def e2e_measure(run, steps, budget_gb, world):
    """Decode through the C `run_kernel` with host buffers: per step H2D of q, K, V,
    block table and lengths from pinned memory, the call, D2H of the output.  The device
    destinations are the resident inputs themselves (the host holds the same bytes), so
    no second device copy of the pool is needed."""
    import torch
    from mx_flash_attn_kernel_opt__b200 import ops
    inp, dev = run.inp, run.dev
    B = inp.batch
    try:
        import psutil
        avail = psutil.virtual_memory().available / 1e9
        budget_gb = min(budget_gb, 0.5 * avail / max(1, world))
    except Exception:
        pass
    pool_bytes = inp.k.numel() * inp.k.element_size() * 2
    per_seq = pool_bytes / B
    limit = B if pool_bytes <= budget_gb * 1e9 else max(1, int(budget_gb * 1e9 // max(per_seq, 1)))
    P = inp.page_size
    if limit < B:
        # host sample: the first sequences and their pages only, on fresh device buffers
        seqs = inp.seq_lens[:limit].cpu()
        npg = ((seqs + P - 1) // P).tolist()
        bt_rows = inp.block_table[:limit].cpu()
        ids = torch.cat([bt_rows[b, :npg[b]] for b in range(limit)]).to(torch.int64)
        width = max(npg)
        bt = torch.zeros(limit, width, dtype=torch.int32)
        pos = 0
        for b in range(limit):
            bt[b, :npg[b]] = torch.arange(pos, pos + npg[b], dtype=torch.int32)
            pos += npg[b]
        dq = [inp.q[:limit].clone(), inp.k.index_select(0, ids.to(dev)),
              inp.v.index_select(0, ids.to(dev)), bt.to(dev), seqs.to(dev)]
        note = f"first {limit} of {B} sequences (host budget {budget_gb:.0f} GB)"
    else:
        dq = [inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens]
        note = "whole workload"
    Bh, width = dq[0].shape[0], dq[3].shape[1]
    nb = dq[1].shape[0]
    if nb != Bh * width:
        # the reference ABI needs pool = batch * row width: pad the table or the pool
        width = max(width, -(-nb // Bh))
        bt2 = torch.zeros(Bh, width, dtype=torch.int32, device=dev)
        bt2[:, :dq[3].shape[1]] = dq[3]
        pad = Bh * width - nb
        k2, v2 = dq[1], dq[2]
        if pad:
            z = torch.zeros((pad,) + tuple(k2.shape[1:]), dtype=k2.dtype, device=dev)
            k2, v2 = torch.cat([k2, z]), torch.cat([v2, z])
        dq = [dq[0], k2, v2, bt2, dq[4]]
    hq = []
    for t in dq:
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        hq.append(h)
    out_d = torch.empty_like(dq[0])
    out_h = torch.empty(out_d.shape, dtype=out_d.dtype, pin_memory=True)
    Hq, D = dq[0].shape[1], dq[0].shape[2]
    Hkv = dq[1].shape[2]
    seqlen_k = int(hq[4].max())
    legacy = torch.cuda.default_stream(dev)
    h2d = sum(t.numel() * t.element_size() for t in hq)
    d2h = out_h.numel() * out_h.element_size()
    kvb = int(hq[4].to(torch.int64).sum()) * Hkv * D * 4

    def one():
        for d, h in zip(dq, hq):
            d.copy_(h, non_blocking=True)
        ops.run_kernel_cabi(dq[0], dq[1], dq[2], out_d, dq[4], dq[3], Bh, seqlen_k, 1, Hq, Hkv,
                            D, P, dq[1].shape[0], 0)
        out_h.copy_(out_d, non_blocking=True)

    n = max(3, min(steps, 20 if h2d < 4e9 else 8))
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
    del hq, out_h
    return {"unit": "GB/s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "steps": n, "ms_per_step": ms, "sample": note, "path": "C run_kernel (ctypes)",
            "_ms": ms, "_kv": float(kvb)}


if __name__ == "__main__":
    main()
