"""Build the tuned-config table (``mla_best_configs_b200.json``) on a B200.

The role of the reference's ``scripts/tune_best.py`` (and its frozen
``mla_best_configs.json``): time candidate configs per shape and keep the
fastest, keyed by shape, dtype and GPU count as ``plan.lookup`` reads it.

    python -m mlc_decode_b200.tune                  # the benchmark shapes
    python -m mlc_decode_b200.tune --shape 64,128,8192,bf16 --out table.json

Candidates are the library default and CTA-pair counts around the SM count
(the tensor-core kernel's only launch knob: how the batch x tile list is cut
into per-pair ranges).  Timing: CUDA events over interleaved repetitions,
median per candidate.  Shapes whose inputs are smaller than twice the 126 MB L2
are timed one call at a time with a 256 MB buffer written between calls (outside
the events), so every call starts with the KV rows out of L2; larger shapes are
timed over back-to-back calls (their inputs do not fit in L2 anyway).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from . import plan
from .decode import MlaDecodeKernel

# (batch, heads, kv_ctx, dtype) per GPU of the benchmark configs: C1, C2, C3
# (ns sweep shape), the C4 head sweep, C5a per GPU at 1/2/4/8 GPUs, C5b per GPU
# at 1/2/4/8 GPUs (sequence split: each GPU holds kv_ctx / N rows).
BENCH_SHAPES = [
    (2, 16, 1024, "fp16"), (64, 128, 8192, "bf16"), (132, 128, 16384, "fp16"),
    (128, 16, 4096, "bf16"), (128, 32, 4096, "bf16"), (128, 64, 4096, "bf16"), (128, 128, 4096, "bf16"),
    (512, 128, 4096, "bf16"), (256, 128, 4096, "bf16"), (64, 128, 4096, "bf16"),
    (1, 128, 131072, "bf16"), (1, 128, 65536, "bf16"), (1, 128, 32768, "bf16"), (1, 128, 16384, "bf16"),
]
DT = {"fp16": torch.float16, "bf16": torch.bfloat16}
L2_BYTES = 126 << 20
FLUSH_BYTES = 256 << 20


def candidates(batch, heads, seqlen_kv):
    cands = [{}]
    for n in (32, 48, 64, 66, 68, 70, 72, 74):
        cands.append({"kernel": "tc", "num_split": n})
    groups = -(-heads // plan.TC_HEADS)
    vb = batch * groups
    for k in (1, 2, 3, 4):
        whole = -(-vb // k)
        if whole <= 74:
            cands.append({"kernel": "tc", "num_split": whole})
    out, seen = [], set()
    for c in cands:
        key = json.dumps(c, sort_keys=True)
        if key not in seen:
            seen.add(key)
            out.append(c)
    return out


def time_shape(batch, heads, seqlen_kv, dtype_name, reps=8, calls=10, cands=None):
    """Median device time per call of each candidate config (default: ``candidates``)
    on seeded inputs of one shape: (candidates, medians in us, index of the fastest)."""
    dt = DT[dtype_name]
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(batch, heads, 512, device=dev, generator=g).to(dt)
    qp = torch.randn(batch, heads, 64, device=dev, generator=g).to(dt)
    kv = torch.randn(batch, seqlen_kv, 1, 512, device=dev, generator=g).to(dt)
    kp = torch.randn(batch, seqlen_kv, 1, 64, device=dev, generator=g).to(dt)
    out = torch.empty_like(q)
    cands = candidates(batch, heads, seqlen_kv) if cands is None else list(cands)
    kerns = [MlaDecodeKernel(batch, heads, 1, seqlen_kv, cfg=c) for c in cands]
    for k in kerns:
        for _ in range(3):
            k(q, qp, kv, kp, out)
    torch.cuda.synchronize()
    in_bytes = sum(x.numel() * x.element_size() for x in (q, qp, kv, kp))
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev) if in_bytes < 2 * L2_BYTES else None
    times = [[] for _ in kerns]
    for r in range(reps):
        order = range(len(kerns)) if r % 2 == 0 else reversed(range(len(kerns)))
        for i in order:
            if flush is None:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(calls):
                    kerns[i](q, qp, kv, kp, out)
                e1.record()
                torch.cuda.synchronize()
                times[i].append(e0.elapsed_time(e1) * 1000.0 / calls)
            else:
                ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                      for _ in range(calls)]
                for e0, e1 in ev:
                    flush.fill_(r & 0xFF)          # evict the inputs from L2
                    e0.record()
                    kerns[i](q, qp, kv, kp, out)
                    e1.record()
                torch.cuda.synchronize()
                times[i].append(statistics.median(e0.elapsed_time(e1) * 1000.0 for e0, e1 in ev))
    med = [statistics.median(t) for t in times]
    best = min(range(len(kerns)), key=lambda i: med[i])
    return cands, med, best


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", action="append", help="batch,heads,kv_ctx,dtype (repeatable)")
    ap.add_argument("--gpus", type=int, default=1, help="GPU count the entries are keyed for")
    ap.add_argument("--out", default=plan.TABLE_PATH)
    a = ap.parse_args()
    shapes = BENCH_SHAPES
    if a.shape:
        shapes = []
        for s in a.shape:
            b, h, ctx, dt = s.split(",")
            shapes.append((int(b), int(h), int(ctx), dt))
    table = plan.load_table(a.out) if os.path.exists(a.out) else {}
    for b, h, ctx, dt in shapes:
        cands, med, best = time_shape(b, h, ctx, dt)
        for c, m in zip(cands, med):
            print(f"b{b} h{h} s{ctx} {dt} {json.dumps(c, sort_keys=True):45s} {m:9.1f} us", flush=True)
        cfg = dict(cands[best])
        cfg["latency_us"] = round(med[best], 1)
        cfg["default_us"] = round(med[0], 1)
        table[plan.table_key(b, h, ctx, dt, a.gpus)] = cfg
        print(f"-> best {cands[best]} {med[best]:.1f} us (default {med[0]:.1f} us)", flush=True)
    with open(a.out, "w") as f:
        json.dump(table, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
