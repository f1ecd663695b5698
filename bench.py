"""Decode-attention benchmark: us per decode step and effective KV TB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
    python bench.py --op quantize [--workload NAME]     # the device KV quantizer, one GPU

One JSON line on rank 0. A "step" is one decode step of one layer over the
workload's KV cache (the kernel plus the split merge), with L2 flushed before
every step: a write of 3 x L2, as the reference times it
(runtime/kvf_host.h:302-330), then a read of 3 x L2 from a second buffer, so
that the step does not also write the flush's dirty lines back to HBM (the
line's "write_flush" gives the step after the write alone). The payload is
2 * rows * (row bytes + 4 * groups) (runtime/kvf_driver.cu:51) over the
stored tokens; value = payload of all ranks / max-over-ranks step time, in
TB/s.

  value   device time of the step, inputs resident in HBM, CUDA events on the
          launching stream
  e2e     the same step through the public API with host buffers, inside the
          timed region: api.Decoder replays the step as a CUDA graph whose
          first kernel reads the queries from pinned host memory and whose
          last writes the output into pinned host memory (sharded workloads:
          copies of the queries in and the output out around the step); the
          KV cache itself stays resident, as a decode cache does
  --impl reference
          the reference's own CPU implementation of the path,
          kvf::reference_attention (runtime/kvf_host.h:202-234, compiled
          unmodified into oracle/_ref), on the host cores, over disjoint
          (sequence, KV head) slices in parallel threads

At N > 1 GPUs (one process per GPU, launched by torch.distributed.run) the
workloads the reference does not shard, the headline among them, run as N
independent replicas (weak scaling, no collective). The two sharded
workloads split one problem over the N GPUs (strong scaling):
  long_gqa_b1_n65536_int4g32_hm         split-KV: each GPU decodes its token
                                        range; the (output, lse) states cross
                                        NVLink inside the split-merge kernel
                                        (--exchange fused; or separate NVLink
                                        kernels, or an NCCL all-gather)
  llama3_70b_b64_n16384_int8g64_tm_p16  KV heads: each GPU owns Hkv/N KV heads of
                                        every sequence; no exchange (the
                                        all-gather of the outputs is timed
                                        separately as "with_output_gather")
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--workload", default=None)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--splits", type=int, default=0, help="override the split count")
    p.add_argument("--exchange", default="fused", choices=["fused", "nvlink", "nccl"],
                   help="split-KV state exchange across GPUs: fused into the split merge over NVLink, separate "
                        "NVLink push/merge kernels, or an NCCL all-gather")
    p.add_argument("--batch", type=int, default=0,
                   help="override the workload's batch (smaller captures for ncu); reported in config")
    p.add_argument("--cpu-sample-s", type=float, default=15.0, help="CPU baseline budget (s)")
    p.add_argument("--op", default="decode", choices=["decode", "quantize"],
                   help="quantize: the device KV quantizer over the workload's K and V rows (one GPU)")
    return p.parse_args()


def measured_peaks() -> dict:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """NVML SM clock and throttle reasons, sampled every 2 ms in a thread."""

    REASONS = {
        0x0000000000000008: "hw_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000080: "hw_power_brake_slowdown",
        0x0000000000000002: "applications_clocks_setting",
    }

    def __init__(self, index: int):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: no clock record
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def record(self) -> dict:
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- reference arm
def reference_step_fn(w, threads: int, sample_seqs=None):
    """One decode step of the reference's CPU path on the same workload:
    kvf::reference_attention over each (sequence, KV head) slice of the
    dequantised cache, slices spread over `threads` threads."""
    import concurrent.futures as cf

    import numpy as np
    import torch

    from kvforge_b200 import workloads
    from oracle import oracle as O

    import dataclasses

    B = w.B if sample_seqs is None else min(w.B, sample_seqs)
    qd, Kd, Vd, seq_lens = workloads.generate(dataclasses.replace(w, B=B), "cpu")
    q = qd.numpy()
    K = Kd.numpy()
    V = Vd.numpy()
    _, _, kd = O.quantize(w.fmt, w.d, w.group, K.reshape(-1, w.d))
    _, _, vd = O.quantize(w.fmt, w.d, w.group, V.reshape(-1, w.d))
    kd = kd.reshape(K.shape)
    vd = vd.reshape(V.shape)
    g = w.H // w.Hkv
    scale = O.scale_f32(w.d)
    slices = []
    for b in range(B):
        nb = w.n if seq_lens is None else int(seq_lens[b])
        for h in range(w.Hkv):
            slices.append((np.ascontiguousarray(q[b : b + 1, h * g : (h + 1) * g]),
                           np.ascontiguousarray(kd[b : b + 1, h : h + 1, :nb]),
                           np.ascontiguousarray(vd[b : b + 1, h : h + 1, :nb])))
    ref_lib = O.Ref.available()
    fn = O.Ref.attention if ref_lib else (lambda a, b_, c, s: O.attention(a, b_, c, s, threads=1))
    pool = cf.ThreadPoolExecutor(max_workers=threads)
    tokens = sum(s[1].shape[2] for s in slices)
    payload = 2 * tokens * (w.d * (16 if w.fmt == 0 else 8 if w.fmt == 1 else 4) // 8 +
                            (0 if w.fmt == 0 else 4 * (w.d // w.group)))

    def step():
        list(pool.map(lambda s: fn(s[0], s[1], s[2], scale), slices))

    return step, payload, ("reference" if ref_lib else "port"), B


def run_reference_arm(args, w, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # A bounded sample: at most 8 sequences of the workload per step.
    step, payload, kind, nseq = reference_step_fn(w, threads, sample_seqs=8)
    for _ in range(max(1, min(args.warmup, 2))):
        step()
    steps = args.steps
    t0 = time.perf_counter()
    step()
    one = time.perf_counter() - t0
    steps = max(1, min(steps, int(60.0 / max(one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    tbs = payload / dt / 1e12
    sample = f"{nseq} of {w.B} sequences per step, all KV heads, dequantised fp32 K/V"
    line = {
        "impl": "reference", "metric": METRIC, "value": tbs, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "us_per_step": dt * 1e6,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic", "config": w.config() | {"sample_sequences": nseq},
        "cpu_baseline": {"value": tbs, "unit": "TB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": tbs, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(w, budget_s: float) -> dict:
    threads = os.cpu_count() or 1
    step, payload, kind, nseq = reference_step_fn(w, threads, sample_seqs=8)
    step()
    t0 = time.perf_counter()
    reps = 0
    while True:
        step()
        reps += 1
        if time.perf_counter() - t0 > min(budget_s, 30.0) or reps >= 20:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": payload / dt / 1e12, "unit": "TB/s", "cores": threads, "kind": kind,
            "us_per_step": dt * 1e6,
            "sample": f"{nseq} of {w.B} sequences, {reps} steps, kvf::reference_attention (fp64) "
                      f"over (sequence, KV head) slices on {threads} threads"}


METRIC = "decode-attn effective KV TB/s (payload bytes / us per step)"


def run_quantize(args, w) -> None:
    """The KV quantizer (kvf_b200_quantize, bit-exact with kvf::quantize,
    runtime/kvf_host.h:72-120) over the workload's logical K and V rows: one
    step quantizes both, with L2 flushed before it. Algorithmic bytes per
    row: 4 * D read, row bytes + 4 * D/G written. The CPU baseline is the
    reference's kvf::quantize (oracle/_ref, else the C restatement) on a
    bounded sample of rows, one thread, as the reference runs it."""
    import ctypes

    import numpy as np
    import torch

    from kvforge_b200 import api, l2flush, workloads
    from kvforge_b200._native import check, lib
    from oracle import oracle as O

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    _, K, V, _ = workloads.generate(w, dev)
    rows = K.numel() // w.d
    rb, gpr = api.row_bytes(w.fmt, w.d), api.groups_per_row(w.fmt, w.d, w.group)
    bufs = []
    for X in (K, V):
        data = torch.empty((rows, rb), dtype=torch.uint8, device=dev)
        meta = torch.empty((rows, max(gpr, 1)), dtype=torch.int32, device=dev)
        bufs.append((X.reshape(rows, w.d), data, meta))
    L = lib()

    def step():
        for X, data, meta in bufs:
            check("kvf_b200_quantize", L.kvf_b200_quantize(w.fmt, w.d, w.group, X.data_ptr(), rows, data.data_ptr(),
                                                           meta.data_ptr() if gpr else None, sptr))

    flush = l2flush.L2Flush(dev)
    for i in range(args.warmup):
        flush(i)
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(0) as clk:
        for i in range(args.steps):
            flush(i)
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    per_row = 4 * w.d + rb + 4 * gpr
    algo = 2 * rows * per_row
    gbs = algo / (ms * 1e-3) / 1e9
    peaks = measured_peaks()

    # CPU: the reference quantizer on a bounded sample of K rows.
    sample = min(rows, 1 << 16)
    Xs = K.reshape(rows, w.d)[:sample].cpu().numpy()
    q = O.Ref.quantize if O.Ref.available() else O.quantize
    q(w.fmt, w.d, w.group, Xs[:1024])
    t0 = time.perf_counter()
    reps = 0
    while reps < 1 or (time.perf_counter() - t0 < min(args.cpu_sample_s, 20.0) and reps < 50):
        q(w.fmt, w.d, w.group, Xs)
        reps += 1
    cpu_s = (time.perf_counter() - t0) / reps
    cpu_gbs = sample * per_row / cpu_s / 1e9
    line = {
        "metric": "KV quantize throughput (algorithmic bytes / us per step)", "value": gbs, "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_step": ms * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {1: "fp32 -> int8", 2: "fp32 -> int4", 0: "fp32 -> f16"}[w.fmt], "data": "synthetic",
        "config": {"workload": w.name, "rows_per_step": 2 * rows, "d": w.d, "group": w.group,
                   "bytes_per_row": per_row, "l2": l2flush.DESCRIPTION},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": None,
                     "peak_source": peaks["source"] + " copy bandwidth (MEASURED_PEAKS.json hbm_gbs)"},
        "cpu_baseline": {"value": cpu_gbs, "unit": "GB/s", "cores": 1,
                         "kind": "reference" if O.Ref.available() else "port",
                         "sample": f"{sample} K rows, {reps} passes, kvf::quantize"},
        "gpu_launches": 2 * args.steps, "clocks": clk.record(), "device_errors": api.device_errors(),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = dist_setup(args.gpus)
    from kvforge_b200 import workloads

    wname = args.workload or workloads.HEADLINE
    w = workloads.WORKLOADS[wname]
    if args.batch:
        import dataclasses

        w = dataclasses.replace(w, B=args.batch)
    if args.op == "quantize":
        if world > 1:
            raise SystemExit("--op quantize runs on one GPU")
        run_quantize(args, w)
        return
    if args.impl == "reference":
        run_reference_arm(args, w, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    import ctypes

    import torch

    from kvforge_b200 import api, l2flush
    from kvforge_b200._native import check, lib

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sharded = world > 1 and w.shard in ("splitkv", "kvheads")
    L = lib()
    g = w.H // w.Hkv
    stream = torch.cuda.current_stream(dev)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    gather_launch = None
    if sharded:
        from kvforge_b200 import sharding

        # One global problem (same seed on every rank), sharded.
        qd, Kd, Vd, seq_lens = workloads.generate(w, dev, seed=w.seed)
        if w.shard == "splitkv":
            sh = sharding.SplitKVDecode(qd, Kd, Vd, fmt=w.fmt, group=w.group, place=w.place, seq_lens=seq_lens,
                                        world=world, rank=rank, splits=args.splits or None, exchange=args.exchange)
        else:
            sh = sharding.HeadShardedDecode(qd, Kd, Vd, fmt=w.fmt, group=w.group, place=w.place, seq_lens=seq_lens,
                                            world=world, rank=rank, splits=args.splits or None)
        del Kd, Vd
        torch.cuda.empty_cache()
        cache, ws, splits = sh.cache, sh.ws, sh.ws.splits
        qd = sh.q
        out = sh.out if w.shard == "splitkv" else sh.out_local
        payload = cache.payload_bytes()

        def launch():
            sh.step()

        if w.shard == "kvheads":
            def gather_launch():
                sh.step(gather=True)

        def api_step():
            sh.step()

        if w.shard == "splitkv":
            parallelism = {
                "fused": f"split-KV over {world} GPUs: split merge stores (out, lse) slices into every GPU over "
                         "NVLink and combines them (one decode + one merge launch)",
                "nvlink": f"split-KV over {world} GPUs: (out, lse) states pushed to peers over NVLink "
                          "(push_state + wait_merge_states kernels)",
                "nccl": f"split-KV over {world} GPUs: NCCL all-gather of (out, lse) + merge_states kernel",
            }[args.exchange]
        else:
            parallelism = f"KV heads over {world} GPUs ({w.Hkv // world} each), no exchange"
        scaling = "strong"
        launches_per_step = (1 if splits <= 1 or "merge=in-kernel" in api.describe(qd, cache, ws) else 2) + (
            {"fused": 0, "nvlink": 2, "nccl": 1}[args.exchange] if w.shard == "splitkv" else 0)
    else:
        qd, Kd, Vd, seq_lens = workloads.generate(w, dev, seed=w.seed + rank)
        cache = api.KVCache.from_logical(Kd, Vd, fmt=w.fmt, group=w.group, place=w.place, seq_lens=seq_lens)
        del Kd, Vd
        torch.cuda.empty_cache()
        splits = args.splits or api.suggest_splits(cache, w.H)
        ws = api.Workspace.allocate(w.B, w.H, w.d, splits, dev)
        out = torch.empty_like(qd)
        payload = cache.payload_bytes()
        args_blk = api.make_args(qd, cache, out, ws)

        def launch():
            check("kvf_b200_decode", L.kvf_b200_decode(ctypes.byref(args_blk), w.fmt, w.d, g, w.place.order,
                                                       int(w.place.paged), sptr))

        def api_step():
            api.decode(qd, cache, out=out, workspace=ws)

        parallelism = f"{world} independent replicas" if world > 1 else "1 GPU"
        scaling = "weak"
        desc = api.describe(qd, cache, ws)
        merge_in_kernel = "merge=in-kernel" in desc
        launches_per_step = 1 if splits <= 1 or merge_in_kernel else 2

    flush = l2flush.L2Flush(dev)
    align_buf = torch.zeros(1, device=dev)

    def prepare(i, clean=True):
        """Untimed before every step: the L2 flush and, with several ranks, a
        device-side all-reduce so that every rank starts the step together
        (a cross-GPU step is as fast as its slowest rank; without this the
        skew between the ranks' flushes would be timed)."""
        flush(i, clean)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(align_buf)

    for i in range(args.warmup):
        prepare(i)
        launch()
    torch.cuda.synchronize()

    # ---- device-timed steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            prepare(i)
            ev[i][0].record(stream)
            launch()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    times_ms = [a.elapsed_time(b) for a, b in ev]
    ms = statistics.mean(times_ms)
    ms_med = statistics.median(times_ms)
    ms_all = max_over_ranks(ms, world)
    errs = api.device_errors()

    # ---- the same steps after the reference's flush alone (a write of
    # 3 x L2, runtime/kvf_host.h:310): the step then also writes the flush's
    # dirty lines back to HBM.
    evw = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    for i in range(args.steps):
        prepare(i, clean=False)
        evw[i][0].record(stream)
        launch()
        evw[i][1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    wf_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in evw), world)

    # ---- with the output all-gather (KV-head sharding only)
    gather_ms = None
    if gather_launch is not None:
        evg = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for i in range(args.warmup):
            prepare(i)
            gather_launch()
        torch.cuda.synchronize()
        barrier(world)
        for i in range(args.steps):
            prepare(i)
            evg[i][0].record(stream)
            gather_launch()
            evg[i][1].record(stream)
        torch.cuda.synchronize()
        barrier(world)
        gather_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in evg), world)

    # ---- end to end through the public API, host buffers: every step copies
    # the queries from pinned host memory, decodes and copies the output back.
    # Unsharded: api.Decoder (the three captured as one CUDA graph, one replay
    # per step); sharded: the sharded object's step between the two copies.
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if not sharded:
        dec = api.Decoder(cache, w.H, splits=splits)
        dec.q_host.copy_(qd.cpu())
        e2e_how = ("api.Decoder, one CUDA graph replay per step: a kernel reads q from pinned host memory "
                   "over PCIe while the decode starts streaming K/V, the kernels write out to pinned host memory")

        def e2e_step():
            dec.replay()
    else:
        q_host = qd.cpu().pin_memory()
        out_host = torch.empty_like(out, device="cpu").pin_memory()
        e2e_how = "H2D of q, sharded step, D2H of out"

        def e2e_step():
            qd.copy_(q_host, non_blocking=True)
            api_step()
            out_host.copy_(out, non_blocking=True)
    for i in range(args.warmup):
        prepare(i)
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    for i in range(args.steps):
        prepare(i)
        ev2[i][0].record(stream)
        e2e_step()
        ev2[i][1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in ev2), world)
    errs |= api.device_errors()

    total_payload = int(sum_over_ranks(float(payload), world))
    value = total_payload / (ms_all * 1e-3) / 1e12
    peaks = measured_peaks()
    achieved_gbs = payload / (ms * 1e-3) / 1e9
    traffic = None
    prof = ROOT / "profiles" / f"{wname}.traffic.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_all, "us_per_step": ms_all * 1e3,
            "us_per_step_median": ms_med * 1e3, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": {0: "f16 KV", 1: "int8 KV", 2: "int4 KV"}[w.fmt] + ", fp32 accumulate",
            "data": "synthetic (seeded N(0,1) on device)",
            "config": w.config() | {"splits": splits, "payload_bytes_per_gpu": payload,
                                    "payload_bytes_total": total_payload,
                                    "l2": l2flush.DESCRIPTION,
                                    "rank_alignment": ("device-side all-reduce before every step, untimed"
                                                       if world > 1 else None),
                                    "parallelism": parallelism},
            "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved_gbs / peaks["hbm_gbs"], "traffic": traffic,
                         "peak_source": peaks["source"] + " copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
                         "timed": "decode kernel + split merge per step"},
            "e2e": {"value": total_payload / (e2e_ms * 1e-3) / 1e12, "unit": "TB/s", "us_per_step": e2e_ms * 1e3,
                    "h2d_bytes_per_step": qd.numel() * 4, "d2h_bytes_per_step": out.numel() * 4,
                    "how": e2e_how},
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_note": "our kernels per timed region (decode, merge when not in-kernel, merge_states); "
                                 "NCCL kernels not counted",
            "clocks": clk.record(),
            "device_errors": errs,
        }
        line["write_flush"] = {"us_per_step": wf_ms * 1e3, "value": total_payload / (wf_ms * 1e-3) / 1e12,
                               "unit": "TB/s", "l2": "the reference's flush alone: a write of 3 x L2"}
        if gather_ms is not None:
            line["with_output_gather"] = {"us_per_step": gather_ms * 1e3,
                                          "value": total_payload / (gather_ms * 1e-3) / 1e12, "unit": "TB/s"}
        if world == 1 and args.cpu_sample_s > 0:
            line["cpu_baseline"] = cpu_baseline(w, args.cpu_sample_s)
        print(json.dumps(line), flush=True)
    if sharded and w.shard == "splitkv":
        sh.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
