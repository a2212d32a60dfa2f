"""Split-count sweep with the combine included (the role of the reference's
``scripts/scan_ns.py``): whole-call device time per ``num_split`` on both kernels.

    python -m mlc_decode_b200.scan_ns                      # the long-cache fp16 config
    python -m mlc_decode_b200.scan_ns --shape 1,128,131072,bf16 --ns 8,16,32,64,74

Default shape: fp16 b132 h128 s16384 (the reference's num_split sweep config), ns in
{1, 2, 4, 8, 16}.  What ``num_split`` means differs by kernel, as it does in the
configs the reference's harness builds:
* CUDA-core kernel (``kernel: "simt"``): KV splits per sequence, the reference's
  meaning (``_split_plan``, even family), each split a CTA per 16 heads, merged by
  the combine launch;
* tensor-core kernel (``kernel: "tc"``): CTA pairs, each owning a contiguous range of
  the batch x tile list; sequences split between pairs are merged in the decode
  launch (up to 3 pieces) or by the combine launch.
The library's default plan is timed beside them.  Timing is ``tune.time_shape``'s:
CUDA events, interleaved repetitions, median; inputs under twice the L2 are timed
one call at a time after a 256 MB write.  Prints one line per config and a JSON
summary line.
"""
from __future__ import annotations

import argparse
import json

from . import tune
from .decode import MlaDecodeKernel


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="132,128,16384,fp16", help="batch,heads,kv_ctx,dtype")
    ap.add_argument("--ns", default="1,2,4,8,16", help="num_split values")
    ap.add_argument("--kernels", default="simt,tc")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--calls", type=int, default=3)
    a = ap.parse_args()
    b, h, ctx, dt = a.shape.split(",")
    b, h, ctx = int(b), int(h), int(ctx)
    ns = [int(x) for x in a.ns.split(",")]
    cands = [{}] + [{"kernel": k, "num_split": n} for k in a.kernels.split(",") for n in ns]
    cands, med, best = tune.time_shape(b, h, ctx, dt, reps=a.reps, calls=a.calls, cands=cands)
    rows = []
    for c, m in zip(cands, med):
        plan = MlaDecodeKernel(b, h, 1, ctx, cfg=c).plan(tune.DT[dt])
        rows.append({"cfg": c or "default", "us": round(m, 1), "kernel": plan["kernel"], "splits": plan["splits"],
                     "launches": plan["launches"]})
        print(f"b{b} h{h} s{ctx} {dt} {json.dumps(c, sort_keys=True) if c else 'default':40s} "
              f"{plan['kernel']:4s} splits {plan['splits']:4d} launches {plan['launches']}  {m:10.1f} us",
              flush=True)
    print(json.dumps({"shape": a.shape, "best": rows[best], "rows": rows}), flush=True)


if __name__ == "__main__":
    main()
