"""Worker of tests/test_multi_gpu.py: one rank per GPU over NCCL.

Checks, on every rank, (a) the batch split (this rank's block of sequences,
no collective) and (b) the sequence split (this rank's part of every KV
cache; float32 partials exchanged over NVLink peer memory or all-gathered,
then merged), both against the float64 oracle.  Exits non-zero on a parity
failure.
"""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from mlc_decode_b200 import MlaDecodeKernel  # noqa: E402
from mlc_decode_b200.dist import SequenceSplitDecoder, batch_shard  # noqa: E402
from oracle import mla_oracle as O  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    ok = True
    try:
        dev = torch.device("cuda", local)
        # (a) batch split
        nb = max(6, world)   # every rank gets at least one sequence
        inputs = O.make_inputs(nb, 128, 1000, "bf16", seed=71)
        sl = batch_shard(nb, rank, world)
        mine = [t[sl].contiguous() for t in inputs]
        q, qp, kv, kp = (t.to(dev) for t in mine)
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[0], 128, device=dev)
        MlaDecodeKernel(q.shape[0], 128, 1, 1000)(q, qp, kv, kp, out, lse)
        torch.cuda.synchronize()
        ref, rl = O.ref_program_f64(*mine)
        res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, rl, "bf16")
        print(f"rank {rank} batch split {res}", flush=True)
        ok &= res["ok"]
        # (b) sequence split, both exchanges (over NVLink peer memory, and the NCCL
        # all-gather), each called three times (both halves of the double buffer).
        # p2p: the one-call path (decode, then one launch that merges this rank's
        # pieces, pushes its rows and merges the peers'), then two calls through the
        # halves (local() into the block, merge() = exchange and merge of the blocks'
        # rows), then one through a caller's combine (the block exchange kernel).
        from mlc_decode_b200 import combine

        cases = [(2, 128, 20000, "bf16", "p2p"), (2, 128, 20000, "bf16", "collective"),
                 (3, 64, 9000, "fp16", "p2p")]
        for b, h, s, dt, exchange in cases:
            inputs = O.make_inputs(b, h, s, dt, seed=72 + h)
            ref, rl = O.ref_program_f64(*inputs)
            dec = SequenceSplitDecoder(b, h, s, exchange=exchange)
            q, qp = inputs[0].to(dev), inputs[1].to(dev)
            kv = inputs[2][:, dec.start:dec.end].contiguous().to(dev)
            kp = inputs[3][:, dec.start:dec.end].contiguous().to(dev)
            routes = ["call"] * 3 if exchange == "collective" or h != 128 else ["call", "call", "halves", "halves",
                                                                                 "call", "combine_fn"]
            for call, route in enumerate(routes):
                out = torch.full((b, h, 512), float("nan"), dtype=q.dtype, device=dev)
                lse = torch.full((b, h), float("nan"), device=dev)
                if route == "call":
                    dec(q, qp, kv, kp, out, lse)
                elif route == "halves":
                    dec.local(q, qp, kv, kp)
                    dec.merge(out, lse)
                else:
                    dec._combine = lambda l_all, o_all, o, l: combine(l_all, o_all, o, l)
                    dec(q, qp, kv, kp, out, lse)
                    dec._combine = combine
                torch.cuda.synchronize()
                res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, rl, dt)
                res["exchange_status"] = dec.exchange_status()
                print(f"rank {rank} sequence split b{b} h{h} {dt} ({exchange}, call {call}, {route}) "
                      f"rows [{dec.start}, {dec.end}) {res}", flush=True)
                ok &= res["ok"] and res["exchange_status"] == 0
            dist.barrier()
            dec.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
