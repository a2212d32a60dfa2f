"""Multi-GPU partitioning host logic on CPU ranks (gloo, world_size 2).

The sequence split (mlc_decode_b200.dist.SequenceSplitDecoder) runs its real
sharding, all-gather and merge path; the per-part decode and the combine are
the oracle's float64 restatements (tests may use the oracle), so the test
checks the partitioning and the merge algebra, not the kernels (the GPU tests
cover those).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlc_decode_b200.dist import batch_shard, seq_shard
from oracle import mla_oracle as O


def test_batch_shard_covers_batch():
    for batch in (1, 2, 7, 64, 512):
        for world in (1, 2, 3, 4, 8):
            parts = [batch_shard(batch, r, world) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == batch
            for a, b in zip(parts, parts[1:]):
                assert a.stop == b.start
            sizes = [p.stop - p.start for p in parts]
            assert max(sizes) - min(sizes) <= 1


def test_seq_shard_whole_tiles():
    for s in (1, 100, 128, 129, 1000, 4096, 131072, 131000):
        for world in (1, 2, 3, 4, 8):
            parts = [seq_shard(s, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == s
            for (a0, a1), (b0, b1) in zip(parts, parts[1:]):
                assert a1 == b0
            for a0, a1 in parts:
                assert (a0 % 128 == 0 or a0 == s) and a1 >= a0
                assert a1 % 128 == 0 or a1 == s
            tiles = [-(-(a1 - a0) // 128) for a0, a1 in parts]
            assert max(tiles) - min(tiles) <= 1


def test_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        seq_shard(100, 2, 2)
    with pytest.raises(ValueError):
        batch_shard(4, -1, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_partial(q, q_pe, kv, k_pe, o, lse):
    po, pl = O.splitkv_partials_f64(q, q_pe, kv, k_pe, [(0, kv.shape[1])])
    o.copy_(torch.from_numpy(po[0]).float())
    lse.copy_(torch.from_numpy(pl[0]).float())


def _oracle_combine(part_lse, part_o, out, lse):
    res, big = O.combine_f64(part_o.numpy(), part_lse.numpy())
    out.copy_(torch.from_numpy(res).to(out.dtype))
    if lse is not None:
        lse.copy_(torch.from_numpy(big).float())


def _rank_main(rank, world, port, cases, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mlc_decode_b200.dist import SequenceSplitDecoder
        for i, (b, h, s, dtype) in enumerate(cases):
            q, qp, kv, kp = O.make_inputs(b, h, s, dtype, seed=i)
            dec = SequenceSplitDecoder(b, h, s, partial_fn=_oracle_partial, combine_fn=_oracle_combine)
            t0, t1 = dec.start, dec.end
            out = torch.empty(b, h, 512, dtype=torch.float32)
            lse = torch.empty(b, h, dtype=torch.float32)
            dec(q, qp, kv[:, t0:t1].contiguous(), kp[:, t0:t1].contiguous(), out, lse)
            ref, rl = O.ref_program_f64(q, qp, kv, kp)
            results.put((rank, i, float(np.abs(out.numpy() - ref).max()),
                         float(np.abs(lse.numpy() - rl).max()), t1 - t0))
    finally:
        dist.destroy_process_group()


def test_sequence_split_gloo_world2():
    """Two CPU ranks: uneven parts, a one-tile sequence (one empty part), bf16 and fp16."""
    cases = [(2, 16, 1000, "bf16"), (1, 8, 100, "fp16"), (1, 4, 640, "bf16")]
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, cases, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    got = {}
    while not results.empty():
        rank, i, err, lerr, rows = results.get()
        got[(rank, i)] = (err, lerr, rows)
    assert len(got) == 2 * len(cases)
    for i, (b, h, s, _) in enumerate(cases):
        assert got[(0, i)][2] + got[(1, i)][2] == s
        for rank in range(2):
            err, lerr, _ = got[(rank, i)]
            # float32 partials merged in float64: float32 rounding only
            assert err < 1e-5, (i, rank, err)
            assert lerr < 1e-5, (i, rank, lerr)
    # the 100-row sequence is one tile: rank 1 holds nothing
    assert got[(1, 1)][2] == 0
