#!/usr/bin/env python3
"""Benchmark of the B200 MLA decode path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (DeepSeek-V3-shaped decode): absorbed-MLA decode, batch 64 per GPU,
128 heads, kv_len 8192, latent 512 + rope 64, bf16, N(0,1) inputs.  A step is
one decode call ``kernel(q, q_pe, kv, k_pe, out)`` (split-KV kernel + LSE
combine).  With N GPUs (torchrun, one rank per GPU) every rank decodes its own
64-sequence batch: the batch is partitioned across GPUs with no collective on
the data path (weak scaling); the step time is the max over ranks.

value       = device time per call (us), CUDA events over exactly K steps
              bracketed by barrier + synchronize; inputs resident in HBM and
              larger than L2 (604 MB per GPU), so no L2 flush is needed.
roofline    = the split-KV kernel against the bound that binds it: its
              algorithmic HBM bytes (b*s*576*2) and flops (2*b*h*s*1088) per
              launch over its mean CUDA-event duration in the same timed
              region, against MEASURED_PEAKS.json's copy bandwidth and the bf16
              tensor rate that applies to the clock the kernel ran at: the
              kernel's clock probe (clock64 / %globaltimer of one CTA, summed
              over the timed calls) gives its SM MHz; within 5 % of the maximum
              clock the burst GEMM rate applies, below it the sustained rate
              (the 1 kW power cap).  frac = max(T_hbm, T_tensor) / kernel time;
              "bound" names the larger term; both fractions are listed.
mla_roofline= the same fraction for the whole call (decode + any combine).
e2e         = the same call through the public API with HOST buffers: pinned
              host->device copies of q, q_pe, kv, k_pe and a device->host read
              of out inside every timed step.
cpu_baseline= the oracle's restatement of the reference torch path
              (baseline_mla.py:167-191) on the host cores, on a bounded batch
              sample, scaled to the full call.

``--fp8`` times the same call over an FP8 (e4m3) latent cache (mla_decode_fp8kv;
the roofline bytes become 512 + 128 per token); ``--paged PAGE_SIZE [--ragged]``
times the paged / variable-length entry point.  ``--seq-split`` times the long-context
sequence split (defaults b1 h128 kv_ctx 131072): under torchrun every rank holds
kv_ctx / N rows of each sequence, a step is its partial decode, the NCCL
all-gather of every rank's (O, LSE) and the LSE merge (``SequenceSplitDecoder``;
scaling "strong": the whole job is one call); with one GPU it is the plain call
on the whole sequence.  The roofline then counts one GPU's share of the rows.

``--impl reference`` times only that reference CPU path (rank 0; other ranks
exit without work) and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MLA decode µs/call + % roofline (b64 h128 s8192 bf16) at 1/2/4/8 B200"
UNIT = "us/call"
L2_BYTES = 126 << 20
FLUSH_BYTES = 256 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=None, help="sequences per GPU (64; --seq-split: 1)")
    ap.add_argument("--heads", type=int, default=128)
    ap.add_argument("--kv-ctx", type=int, default=None, help="KV rows per sequence (8192; --seq-split: 131072)")
    ap.add_argument("--dtype", choices=["bf16", "fp16"], default="bf16")
    ap.add_argument("--kernel", choices=["auto", "tc", "simt"], default="auto")
    ap.add_argument("--num-split", type=int, default=0)
    ap.add_argument("--combine-groups", type=int, default=0,
                    help="config key combine_groups (>= 2: wide splits merged by a separate combine launch)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="budget of host-core time for the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--paged", type=int, default=0, metavar="PAGE_SIZE",
                    help="decode through mla_decode_paged with KV in shuffled pages of this many rows")
    ap.add_argument("--fp8", action="store_true",
                    help="decode through mla_decode_fp8kv: e4m3 latent cache (scale 1/16), rope in --dtype")
    ap.add_argument("--ragged", action="store_true",
                    help="with --paged: per-sequence lengths drawn uniformly from [1, kv_ctx] (seeded)")
    ap.add_argument("--seq-exchange", choices=["auto", "p2p", "collective"], default="auto",
                    help="--seq-split under torchrun: the exchange of the ranks' (O, LSE) blocks")
    ap.add_argument("--seq-split", action="store_true",
                    help="long-context sequence split: every sequence's KV rows split across the ranks, "
                         "(O, LSE) all-gathered over NCCL and merged")
    a = ap.parse_args()
    if a.batch is None:
        a.batch = 1 if a.seq_split else 64
    if a.kv_ctx is None:
        a.kv_ctx = 131072 if a.seq_split else 8192
    if a.seq_split and (a.paged or a.fp8):
        ap.error("--seq-split takes neither --paged nor --fp8")
    return a


def workload_name(a):
    name = f"mla_decode b{a.batch}/gpu h{a.heads} s{a.kv_ctx} {a.dtype} (dim 512+64, kv_heads 1)"
    if a.paged:
        name += f", paged KV ({a.paged}-row pages" + (", ragged lengths)" if a.ragged else ")")
    if a.fp8:
        name += ", FP8 (e4m3) latent KV cache"
    if a.seq_split:
        name = f"mla_decode b{a.batch} h{a.heads} s{a.kv_ctx} {a.dtype} (dim 512+64, kv_heads 1), "
        how = {"collective": "all-gathered over NCCL",
               "p2p": "merged per GPU and pushed row by row over NVLink peer memory",
               "auto": "merged per GPU and pushed row by row over NVLink peer memory (NCCL all-gather where "
                       "peers are not reachable)"}
        name += (f"KV rows split across {a.gpus} GPU(s), (O, LSE) {how[a.seq_exchange]} and merged"
                 if a.gpus > 1 else "whole sequence on one GPU (the sequence split's 1-GPU point)")
    return name


def config_of(a, world, kv_bytes=None, flushed=None):
    """The `config` object of the JSON line: the same keys in both arms."""
    if kv_bytes is None:
        per_row = 512 * (1 if a.fp8 else 2) + 64 * 2
        kv_bytes = a.batch * a.kv_ctx * per_row // (world if a.seq_split else 1)
    if flushed is None:
        flushed = kv_bytes < 2 * L2_BYTES
    return {"workload": workload_name(a), "batch_per_gpu": a.batch, "global_batch": a.batch * (1 if a.seq_split else world),
            "heads": a.heads, "kv_ctx": a.kv_ctx, "kernel": a.kernel, "num_split": a.num_split or "auto",
            "parallelism": (f"sequence split over {world} GPU(s): exchange of (O, LSE) ({a.seq_exchange}), LSE merge"
                            if a.seq_split and world > 1 else f"batch split over {world} GPU(s), no collective"),
            "l2": ("inputs (KV+K_pe %.0f MB per GPU) larger than the 126 MB L2; no flush" % (kv_bytes / 1e6)
                   if not flushed else
                   "inputs (KV+K_pe %.0f MB per GPU) under twice the 126 MB L2: a 256 MB buffer "
                   "written before every step, outside its events" % (kv_bytes / 1e6))}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, source="fallback")


def algorithmic(b, h, s, fp8=False):
    # bytes: the latent (2 bytes a dim, or 1 for the e4m3 cache) and rope rows of every KV token
    return b * s * (512 * (1 if fp8 else 2) + 64 * 2), 2.0 * b * h * s * (576 + 512)


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def mark(self, begin):
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = time.mktime(time.strptime(parts[1].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                    rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        inside = [r for r in rows if self.t0 - 1.0 <= r[0] <= self.t1 + 1.0] or rows
        reasons = sorted({self.NAMES[i] for r in inside for i, v in enumerate(r[3]) if v == "Active"})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": inside[0][2],
                "reasons": reasons, "samples": len(inside)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference torch path restated by the oracle, on host cores
# ---------------------------------------------------------------------------
def cpu_time_per_call(a, budget_s, steps=None):
    """Median seconds of ref_program_torch on a batch sample, scaled to the full call."""
    import torch

    from oracle.mla_oracle import make_inputs, ref_program_torch

    torch.set_num_threads(os.cpu_count() or 1)
    probe = make_inputs(1, a.heads, a.kv_ctx, a.dtype, seed=0)
    ref_program_torch(*probe)
    t = time.perf_counter()
    ref_program_torch(*probe)
    t1 = max(time.perf_counter() - t, 1e-4)
    reps = steps if steps is not None else 3
    bs = int(max(1, min(a.batch, budget_s / (reps + 1) / t1)))
    inp = make_inputs(bs, a.heads, a.kv_ctx, a.dtype, seed=0)
    ref_program_torch(*inp)
    times = []
    for _ in range(reps):
        t = time.perf_counter()
        ref_program_torch(*inp)
        times.append(time.perf_counter() - t)
    return times, bs, torch.get_num_threads()


def run_reference(a, rank):
    if rank != 0:
        return
    warm = max(0, a.warmup)
    times, bs, cores = cpu_time_per_call(a, a.cpu_seconds * 8, steps=a.steps + min(warm, 3))
    times = times[min(warm, 3):] or times
    us = statistics.median(times) * 1e6 * (a.batch / bs)
    sample = (f"{bs} of {a.batch} sequences per step (same heads/kv_ctx/dtype), median of "
              f"{len(times)} steps, scaled x{a.batch / bs:g} to the full call")
    line = {"impl": "reference", "metric": METRIC, "value": round(us, 3), "unit": UNIT,
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(us / 1000, 3), "higher_is_better": False,
            "scaling": "strong" if a.seq_split else "weak",
            "vs_baseline": None, "dtype": a.dtype, "data": "synthetic N(0,1), seeded",
            "config": config_of(a, a.gpus), "arm": "reference CPU path (torch on host cores)",
            "cpu_baseline": {"value": round(us, 3), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(us, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def traffic_from_profiles(a):
    """Per-launch DRAM bytes of the split-KV kernel from a committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    ent = d.get(f"b{a.batch}_h{a.heads}_s{a.kv_ctx}_{a.dtype}_{a.kernel}") or \
        d.get(f"b{a.batch}_h{a.heads}_s{a.kv_ctx}_{a.dtype}")
    return None if ent is None else ent.get("dram_bytes_per_launch")


def read_probe(obj, dev, dtype):
    """(cycles, ns, calls) of the decode kernel's clock probe, or None (CUDA-core kernel)."""
    if obj is None or not hasattr(obj, "clock_probe"):
        return None
    try:
        return obj.clock_probe(dev, dtype)
    except Exception:  # noqa: BLE001 - the probe is informational
        return None


def kernel_clock(p0, p1, sm_max):
    """SM clock the decode kernel ran at inside the timed region, from its probe."""
    if p0 is None or p1 is None or p1[2] <= p0[2] or p1[1] <= p0[1]:
        return None
    mhz = (p1[0] - p0[0]) / (p1[1] - p0[1]) * 1000.0
    return {"sm_mhz": round(mhz, 1), "calls": p1[2] - p0[2],
            "of_max": round(mhz / sm_max, 4) if sm_max else None,
            "how": "clock64 and %globaltimer over one CTA's whole run, every call, summed"}


def run_ours(a, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from mlc_decode_b200 import MlaDecodeKernel, MlaPagedDecodeKernel

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    b, h, s = a.batch, a.heads, a.kv_ctx
    tdt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    cfg = {"kernel": a.kernel}
    if a.num_split:
        cfg["num_split"] = a.num_split
    if a.combine_groups:
        cfg["combine_groups"] = a.combine_groups

    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    q = torch.randn(b, h, 512, device=dev, generator=g).to(tdt)
    q_pe = torch.randn(b, h, 64, device=dev, generator=g).to(tdt)
    lens = [s] * b
    if a.paged:
        # KV rows scattered over shuffled pages (the serving layout), block table per sequence
        if a.ragged:
            gl = torch.Generator().manual_seed(99 + rank)
            lens = [int(x) for x in torch.randint(1, s + 1, (b,), generator=gl)]
        ps = a.paged
        npg = [-(-L // ps) for L in lens]
        num_pages = sum(npg)
        perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(7 + rank))
        table = torch.zeros(b, max(npg), dtype=torch.int32)
        k = 0
        for bb in range(b):
            for i in range(npg[bb]):
                table[bb, i] = int(perm[k])
                k += 1
        kv = torch.randn(num_pages, ps, 1, 512, device=dev, generator=g).to(tdt)
        k_pe = torch.randn(num_pages, ps, 1, 64, device=dev, generator=g).to(tdt)
        table = table.to(dev)
        seqlens = torch.tensor(lens, dtype=torch.int32, device=dev)
        pkern = MlaPagedDecodeKernel(b, h, s, cfg=cfg)

        class _Paged:
            def __call__(self, q_, qp_, kv_, kp_, out_):
                pkern(q_, qp_, kv_, kp_, seqlens, out_, block_table=table)

            splitkv = __call__

            def combine_ws(self, out_):
                pass

        kern = _Paged()
        probe_obj = pkern
        launches = 3
    elif a.fp8:
        base = MlaDecodeKernel(b, h, 1, s, cfg=cfg)
        # N(0,1) latent rows stored as e4m3 codes of kv / (1/16)
        kv = (torch.randn(b, s, 1, 512, device=dev, generator=g) * 16).clamp(-448, 448).to(torch.float8_e4m3fn)
        k_pe = torch.randn(b, s, 1, 64, device=dev, generator=g).to(tdt)

        class _Fp8:
            def __call__(self, q_, qp_, kv_, kp_, out_):
                base.decode_fp8(q_, qp_, kv_, kp_, 1.0 / 16, out_)

            splitkv = __call__

            def combine_ws(self, out_):
                pass

        kern = _Fp8()
        probe_obj = base
        launches = base.launches_per_call(tdt)
    elif a.seq_split and world > 1:
        from mlc_decode_b200.dist import SequenceSplitDecoder

        # every rank decodes the same queries against its own rows of the sequences
        gq = torch.Generator(device=dev).manual_seed(1234)
        q = torch.randn(b, h, 512, device=dev, generator=gq).to(tdt)
        q_pe = torch.randn(b, h, 64, device=dev, generator=gq).to(tdt)
        dec = SequenceSplitDecoder(b, h, s, cfg=cfg, exchange=a.seq_exchange)
        lens = [dec.local_len] * b
        kv = torch.randn(b, dec.local_len, 1, 512, device=dev, generator=g).to(tdt)
        k_pe = torch.randn(b, dec.local_len, 1, 64, device=dev, generator=g).to(tdt)

        class _Seq:
            # A timed step is the whole call: over NVLink peer memory two launches
            # (this rank's decode, then one launch that merges its rows, stores them
            # into the peers' buffers and merges theirs); over the all-gather the
            # decode and its combine, the collective and the merge.
            def __call__(self, q_, qp_, kv_, kp_, out_):
                dec(q_, qp_, kv_, kp_, out_)

            splitkv = __call__

            def combine_ws(self, out_):
                pass

        kern = _Seq()
        probe_obj = dec.kernel
        p2p = dec._use_p2p(dev)
        launches = 2 if p2p else (dec.kernel.launches_per_call(tdt) if dec.kernel is not None else 0) + 1
    else:
        kern = MlaDecodeKernel(b, h, 1, s, cfg=cfg)
        probe_obj = kern
        kv = torch.randn(b, s, 1, 512, device=dev, generator=g).to(tdt)
        k_pe = torch.randn(b, s, 1, 64, device=dev, generator=g).to(tdt)
        launches = kern.launches_per_call(tdt)
    out = torch.empty_like(q)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(max(3, a.warmup)):
        kern(q, q_pe, kv, k_pe, out)
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    clocks.start()
    K = a.steps
    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # KV rows on this GPU smaller than twice the L2: write a 256 MB buffer before every
    # step, outside per-step events, so that no step finds its rows in L2
    kv_bytes = kv.numel() * kv.element_size() + k_pe.numel() * k_pe.element_size()
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev) if kv_bytes < 2 * L2_BYTES else None
    ev_s = [torch.cuda.Event(enable_timing=True) for _ in range(K)] if flush is not None else None
    ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(K)] if flush is not None else None
    barrier()
    torch.cuda.synchronize()
    probe0 = read_probe(probe_obj, dev, tdt)
    clocks.mark(True)
    start.record()
    for i in range(K):
        if flush is not None:
            flush.fill_(i & 0xFF)
            ev_s[i].record()
        ev_a[i].record()
        kern.splitkv(q, q_pe, kv, k_pe, out)
        ev_b[i].record()
        kern.combine_ws(out)
        if flush is not None:
            ev_e[i].record()
    end.record()
    torch.cuda.synchronize()
    clocks.mark(False)
    probe1 = read_probe(probe_obj, dev, tdt)
    barrier()
    clk = clocks.stop()
    total_ms = (start.elapsed_time(end) if flush is None else
                sum(ev_s[i].elapsed_time(ev_e[i]) for i in range(K)))
    dec_ms = [ev_a[i].elapsed_time(ev_b[i]) for i in range(K)]
    t = torch.tensor([total_ms, statistics.mean(dec_ms)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, dec_mean_ms = float(t[0]), float(t[1])
    us_call = total_ms * 1000.0 / K
    dec_us = dec_mean_ms * 1000.0
    if a.seq_split and world > 1:
        # the dominant kernel's time, for the roofline: this rank's decode launch alone
        # (the same decode kernel the call launches first), timed after the timed
        # region with the same flush before each launch
        dec_us = seq_decode_us(dec, q, q_pe, kv, k_pe, out, flush, min(K, 50), dev, world)

    # ---- e2e through the public API with host buffers ------------------------
    hq, hqp, hkv, hkp = (x.cpu().pin_memory() for x in (q, q_pe, kv, k_pe))
    hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    dq, dqp, dkv, dkp = (torch.empty_like(x) for x in (q, q_pe, kv, k_pe))
    E = max(3, min(a.e2e_steps, K))

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        dqp.copy_(hqp, non_blocking=True)
        dkv.copy_(hkv, non_blocking=True)
        dkp.copy_(hkp, non_blocking=True)
        kern(dq, dqp, dkv, dkp, out)
        hout.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(E):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_us = float(te[0]) * 1000.0 / E
    h2d = sum(x.numel() * x.element_size() for x in (hq, hqp, hkv, hkp))
    d2h = hout.numel() * hout.element_size()
    del hq, hqp, hkv, hkp, dq, dqp, dkv, dkp

    if rank != 0:
        return
    peaks = load_peaks()
    bytes_alg, flops_alg = algorithmic(1, h, sum(lens), a.fp8)
    achieved = bytes_alg / (dec_us * 1e-6) / 1e9                 # GB/s
    achieved_tc = flops_alg / (dec_us * 1e-6) / 1e12             # TFLOP/s
    sm_max = (clk or {}).get("sm_max_mhz") or 1965.0
    kclk = kernel_clock(probe0, probe1, sm_max)
    # Which tensor peak applies is read off the clock the kernel actually ran at:
    # within 5 % of the maximum SM clock the part was not power-capped during the
    # timed region (a short run), so the burst GEMM rate applies; below it, the
    # sustained rate under the 1 kW cap.  Without a probe (CUDA-core kernel): burst
    # for a timed region under 50 ms, else sustained.
    if kclk is not None:
        sustained = kclk["sm_mhz"] < 0.95 * sm_max
    else:
        sustained = total_ms > 50.0
    tc_peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    t_hbm_us = bytes_alg / (peaks["hbm_gbs"] * 1e9) * 1e6
    t_tc_us = flops_alg / (tc_peak * 1e12) * 1e6
    t_roof_us = max(t_hbm_us, t_tc_us)
    tensor_bound = t_tc_us > t_hbm_us and not a.fp8   # (FP8 QK^T: not the bf16 tensor rate)
    peak_kind = "sustained" if sustained else "burst"
    line = {
        "metric": METRIC, "value": round(us_call, 3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": a.warmup, "ms_per_step": round(us_call / 1000.0, 5), "higher_is_better": False,
        "scaling": "strong" if a.seq_split else "weak", "vs_baseline": None, "dtype": a.dtype,
        "data": "synthetic N(0,1), seeded, generated on device",
        "config": config_of(a, world, kv_bytes, flush is not None), "arm": "B200 CUDA kernels",
        "roofline": {"bound": "tensor" if tensor_bound else "hbm",
                     "achieved": round(achieved_tc if tensor_bound else achieved, 1),
                     "peak": tc_peak if tensor_bound else peaks["hbm_gbs"],
                     "unit": "TFLOP/s" if tensor_bound else "GB/s",
                     "frac": round(t_roof_us / dec_us, 4),
                     "peak_kind": peak_kind,
                     "hbm": {"achieved_gbs": round(achieved, 1), "peak_gbs": peaks["hbm_gbs"],
                             "frac": round(achieved / peaks["hbm_gbs"], 4)},
                     "tensor": {"achieved_tflops": round(achieved_tc, 1), "peak_tflops": tc_peak,
                                "peak_kind": peak_kind, "frac": round(achieved_tc / tc_peak, 4),
                                "burst_peak_tflops": peaks["bf16_tflops"],
                                "sustained_peak_tflops": peaks["bf16_tflops_sustained"]},
                     "traffic": None if (a.paged or a.fp8 or a.seq_split) else traffic_from_profiles(a),
                     "kernel": ("paged decode call (plan + decode + combine)" if a.paged else
                                "FP8-KV split-KV decode kernel" if a.fp8 else
                                "decode kernel of this GPU's KV rows (the first of the call's launches)"
                                if a.seq_split and world > 1 else
                                "split-KV decode kernel"),
                     "kernel_us": round(dec_us, 3), "peak_source": peaks["source"],
                     "kernel_clock": kclk,
                     "kernel_kcycles": (round(dec_us * kclk["sm_mhz"] / 1000.0, 1) if kclk else None)},
        "mla_roofline": {"t_roof_us": round(t_roof_us, 3), "peak_kind": peak_kind,
                         "frac": round(t_roof_us / us_call, 4),
                         "t_hbm_us": round(t_hbm_us, 3), "t_tensor_us": round(t_tc_us, 3),
                         "hbm_bytes": bytes_alg, "flops": flops_alg,
                         "peaks": {"hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"],
                                   "bf16_tflops_sustained": peaks["bf16_tflops_sustained"],
                                   "source": peaks["source"]}},
        "e2e": {"value": round(e2e_us, 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": E},
        "gpu_launches": K * launches,
        "clocks": clk,
    }
    if a.paged or a.seq_split:
        line["config"]["kv_rows_total" if a.paged else "kv_rows_per_gpu"] = sum(lens)
    if world == 1 and not a.no_cpu_baseline and not a.paged and not a.fp8:
        times, bs, cores = cpu_time_per_call(a, a.cpu_seconds)
        cpu_us = statistics.median(times) * 1e6 * (b / bs)
        line["cpu_baseline"] = {"value": round(cpu_us, 3), "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": f"{bs} of {b} sequences, median of {len(times)} runs, "
                                          f"scaled x{b / bs:g} to the full call"}
    print(json.dumps(line), flush=True)


def seq_decode_us(dec, q, q_pe, kv, k_pe, out, flush, n, dev, world):
    """Mean device time of the sequence split's decode launch on this rank's KV rows
    (MlaDecodeKernel.splitkv: the decode kernel alone), max over ranks."""
    import torch
    import torch.distributed as dist

    k = dec.kernel
    if k is None:
        return 0.0
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for i in range(n):
        if flush is not None:
            flush.fill_(i & 0xFF)
        ev[i][0].record()
        k.splitkv(q, q_pe, kv, k_pe, out)
        ev[i][1].record()
    torch.cuda.synchronize()
    t = torch.tensor([statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev) * 1000.0], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def main():
    a = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(a, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
