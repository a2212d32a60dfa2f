"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is importable:

    python tests/golden/gen_golden.py --ref <path to NiseAzaka/mlc_decode checkout>

It imports the reference's own ``baseline_mla.ref_program``
(baseline_mla.py:167-191) and ``mla_decode._split_plan`` (mla_decode.py:9-30)
and writes:

* ``ref_program.npz`` -- for each case, SHA-256 digests of the seeded inputs
  (so a test can prove it regenerated the same inputs), the reference output
  on float64 upcasts of the inputs (stored as float32), the reference output in the native input
  dtype, and the float64 log-sum-exp of the same scaled scores (torch
  ``logsumexp``; the reference has no LSE output, so this defines the LSE
  oracle).
* ``split_plan.json`` -- ``_split_plan`` on a grid of (kv_ctx, num_split,
  block_N, spread), including the tail cases the reference documents.
* ``ref_program_grouped.npz`` / ``ref_program_grouped_cases.json`` -- the same
  for kv_head_num > 1 (``ref_program`` groups query heads over KV heads,
  baseline_mla.py:179-189, although the reference's kernels assert
  kv_head_num == 1), inputs from ``make_inputs_ext`` with q_len = 1.

``--only grouped`` rewrites just the grouped files.

Nothing on the GPU box runs this script: the fixtures it writes are committed.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.mla_oracle import make_inputs, make_inputs_ext  # noqa: E402

# (name, dtype, batch, heads, kv_ctx, seed, scale)
CASES = [
    ("c1_fp16_b2_h16_s1024", "fp16", 2, 16, 1024, 0, 1.0),       # the CPU-runnable reference case
    ("c1_fp16_b2_h16_s1024_x0.1", "fp16", 2, 16, 1024, 0, 0.1),  # check_mla.py distribution
    ("tail_fp16_s7", "fp16", 1, 16, 7, 1, 1.0),
    ("tail_fp16_s33", "fp16", 1, 16, 33, 2, 1.0),
    ("tail_fp16_s3000", "fp16", 1, 16, 3000, 3, 1.0),
    ("tail_fp16_s3008", "fp16", 1, 16, 3008, 4, 1.0),
    ("tail_fp16_s4095", "fp16", 1, 16, 4095, 5, 1.0),
    ("tail_bf16_s4096", "bf16", 1, 16, 4096, 6, 1.0),
    ("s1_bf16_h16", "bf16", 2, 16, 1, 7, 1.0),
    ("h32_bf16_s300", "bf16", 2, 32, 300, 8, 1.0),
    ("h64_bf16_s513", "bf16", 1, 64, 513, 9, 1.0),
    ("h128_bf16_s640", "bf16", 2, 128, 640, 10, 1.0),
    ("h128_fp16_s1000_x0.1", "fp16", 1, 128, 1000, 11, 0.1),
    ("bench_bf16_b1_h128_s8192", "bf16", 1, 128, 8192, 12, 1.0),   # one sequence of the bench call
    ("longcache_fp16_b1_h128_s16384", "fp16", 1, 128, 16384, 13, 1.0),
]

# (name, dtype, batch, heads, kv_heads, kv_ctx, seed): grouped KV heads
GROUPED_CASES = [
    ("grouped_bf16_b2_h128_kv2_s300", "bf16", 2, 128, 2, 300, 20),
    ("grouped_fp16_b1_h64_kv4_s129", "fp16", 1, 64, 4, 129, 21),
    ("grouped_bf16_b2_h32_kv8_s77", "bf16", 2, 32, 8, 77, 22),
    ("grouped_bf16_b1_h256_kv2_s640", "bf16", 1, 256, 2, 640, 23),
]

# (kv_ctx, num_split, block_N, spread) grid for _split_plan.
PLAN_CTX = [1, 7, 31, 32, 33, 63, 64, 65, 1000, 2048, 3000, 3008, 4095, 4096,
            8192, 16384, 32768, 65536, 131072]
PLAN_NS = [1, 2, 3, 7, 64, 104, 148, 208, 296, 312, 1024]
PLAN_BN = [16, 32, 64, 128]


def digest(t):
    return hashlib.sha256(t.contiguous().view(-1).view(__import__("torch").uint8).numpy().tobytes()).hexdigest()


def gen_grouped(baseline_mla):
    import torch

    arrays, meta = {}, []
    for name, dtype, b, h, kvh, s, seed in GROUPED_CASES:
        q, q_pe, kv, k_pe = make_inputs_ext(b, 1, h, kvh, s, dtype, seed)
        q, q_pe = q[:, 0].contiguous(), q_pe[:, 0].contiguous()
        with torch.no_grad():
            out64 = baseline_mla.ref_program(q.double(), q_pe.double(), kv.double(), k_pe.double())
        arrays[f"{name}/out64"] = out64.float().numpy()
        meta.append({"name": name, "dtype": dtype, "batch": b, "heads": h, "kv_heads": kvh, "kv_ctx": s,
                     "seed": seed, "sha256": [digest(t) for t in (q, q_pe, kv, k_pe)]})
    np.savez_compressed(os.path.join(HERE, "ref_program_grouped.npz"), **arrays)
    with open(os.path.join(HERE, "ref_program_grouped_cases.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(f"wrote {len(meta)} grouped ref_program cases")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("--only", choices=["grouped"], default=None)
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.ref))
    import torch
    import baseline_mla  # the reference oracle
    import mla_decode    # the reference planner

    gen_grouped(baseline_mla)
    if args.only == "grouped":
        return

    arrays = {}
    meta = []
    for name, dtype, b, h, s, seed, scale in CASES:
        q, q_pe, kv, k_pe = make_inputs(b, h, s, dtype, seed, scale)
        with torch.no_grad():
            out64 = baseline_mla.ref_program(q.double(), q_pe.double(), kv.double(), k_pe.double())
            outn = baseline_mla.ref_program(q, q_pe, kv, k_pe)
            qf = torch.cat([q.double(), q_pe.double()], dim=-1)
            kf = torch.cat([kv.double()[:, :, 0], k_pe.double()[:, :, 0]], dim=-1)
            lse = torch.logsumexp(torch.einsum("bhd,bsd->bhs", qf, kf) * (576 ** -0.5), dim=-1)
        arrays[f"{name}/out64"] = out64.float().numpy()  # float32 storage of the float64 result
        arrays[f"{name}/out_native"] = outn.float().numpy()
        arrays[f"{name}/lse64"] = lse.numpy()
        # the native-dtype output of a long sequence depends on torch's CPU thread
        # count (reduction order): record it so a test can replay it exactly
        meta.append({"name": name, "dtype": dtype, "batch": b, "heads": h, "kv_ctx": s,
                     "seed": seed, "scale": scale, "threads": torch.get_num_threads(),
                     "sha256": [digest(t) for t in (q, q_pe, kv, k_pe)]})
    np.savez_compressed(os.path.join(HERE, "ref_program.npz"), **arrays)
    with open(os.path.join(HERE, "ref_program_cases.json"), "w") as f:
        json.dump(meta, f, indent=1)

    plans = []
    for s in PLAN_CTX:
        for ns in PLAN_NS:
            for bn in PLAN_BN:
                for spread in (False, True):
                    plans.append([s, ns, bn, int(spread), list(mla_decode._split_plan(s, ns, bn, spread))])
    with open(os.path.join(HERE, "split_plan.json"), "w") as f:
        json.dump(plans, f)
    print(f"wrote {len(meta)} ref_program cases, {len(plans)} split plans")


if __name__ == "__main__":
    main()
