"""The sequence split's fused exchange-and-merge launch on one GPU.

mla_seqsplit_decode decodes this rank's KV part, then one launch merges its rows
(from the decode kernel's pieces when a sequence was split between many CTA
pairs), stores each row into every peer's gather buffer as (value, call number)
words, polls for the peers' rows and merges them.  Launches that wait on one another never run
on one GPU, so the peers here are emulated without any waiting launch:

* world 1: no peers; the output must be the decode of the whole part;
* world 2: the second rank's rows are written into the first rank's buffer,
  tagged with the call's number, before the first rank's launch (as the second
  rank's launch would have), so every wait is already satisfied; the output must
  be the decode over both parts, and the first rank's rows must have landed in the
  second buffer with this call's number;
* a peer that never delivers: its words never carry the call's number, the
  launch gives up after its time limit (2 s) and the status word says 0x201; the
  context stays usable.

All against the float64 oracle, on both call parities.
"""
import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

DIM = 512


def _layout(world, b, h):
    bh = b * h
    rows_pad = -(-bh // 64) * 64
    chunk = bh * DIM + rows_pad
    header = -(-2 * world * chunk * 4 // 256) * 256
    ll_rows = header + 256
    ll_lse = ll_rows + 2 * world * rows_pad * DIM * 8
    return chunk, header, rows_pad, ll_rows, ll_lse


def _buffer(world, b, h, dev):
    from mlc_decode_b200 import capi

    n = capi.seqsplit_buffer_bytes(world, b, h)
    _, _, rows_pad, _, ll_lse = _layout(world, b, h)
    assert n == ll_lse + 2 * world * rows_pad * 8
    return torch.zeros(n, dtype=torch.uint8, device=dev)


def _block(buf, world, b, h, par, r):
    chunk = _layout(world, b, h)[0]
    f = buf[: 2 * world * chunk * 4].view(torch.float32).view(2, world, chunk)[par, r]
    return f[: b * h * DIM].view(b, h, DIM), f[b * h * DIM: b * h * (DIM + 1)].view(b, h)


def _words(buf, world, b, h, par, r):
    """Rank r's row words [b*h, 512, 2] and LSE words [b*h, 2] of parity par:
    (value bits, call number) pairs."""
    _, _, rows_pad, ll_rows, ll_lse = _layout(world, b, h)
    rows = buf[ll_rows: ll_lse].view(torch.int32).view(2, world, rows_pad, DIM, 2)[par, r, : b * h]
    lse = buf[ll_lse:].view(torch.int32).view(2, world, rows_pad, 2)[par, r, : b * h]
    return rows, lse


def _deliver(buf, world, b, h, par, r, o, l, epoch):
    """Write rank r's (O, LSE) into buf's words as rank r's launch would."""
    rows, lse = _words(buf, world, b, h, par, r)
    rows[..., 0] = o.reshape(b * h, DIM).view(torch.int32)
    rows[..., 1] = epoch
    lse[:, 0] = l.reshape(b * h).view(torch.int32)
    lse[:, 1] = epoch


def _status(buf, world, b, h):
    header = _layout(world, b, h)[1]
    return int(buf[header + 68: header + 72].view(torch.int32).item())


def _ref(inputs):
    return O.ref_program_f64(*inputs)


@pytest.mark.parametrize("cfg", [None, {"kernel": "simt", "num_split": 3}], ids=["auto", "simt"])
@pytest.mark.parametrize("b,h,s,dt", [(1, 128, 20000, "bf16"), (2, 128, 3000, "fp16"), (3, 64, 5000, "bf16"),
                                     (1, 256, 9000, "bf16")])
def test_world1_matches_whole_decode(b, h, s, dt, cfg, cuda):
    """auto: one sequence split between many CTA pairs, merged from its pieces in the
    exchange launch (b1), or rows the decode kernel wrote whole; simt: the CUDA-core
    kernel and its combine write the block, the exchange launch takes it from there."""
    from mlc_decode_b200 import MlaDecodeKernel

    inputs = O.make_inputs(b, h, s, dt, seed=300 + b)
    ref, rl = _ref(inputs)
    q, qp, kv, kp = (t.to(cuda) for t in inputs)
    buf = _buffer(1, b, h, cuda)
    k = MlaDecodeKernel(b, h, 1, s, cfg=cfg)
    for epoch in (1, 2, 3):
        out = torch.full((b, h, DIM), float("nan"), dtype=q.dtype, device=cuda)
        lse = torch.full((b, h), float("nan"), device=cuda)
        k.seqsplit(q, qp, kv, kp, out, lse, [buf.data_ptr()], 1, 0, epoch)
        torch.cuda.synchronize()
        res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, rl, dt)
        assert res["ok"], (epoch, res)
        assert _status(buf, 1, b, h) == 0


@pytest.mark.parametrize("b,h,s,dt", [(1, 128, 40000, "bf16"), (3, 64, 9000, "fp16"), (2, 256, 6000, "bf16")])
def test_world2_emulated_peer(b, h, s, dt, cuda):
    """Rank 0's launch against a peer whose rows and flags are already in place."""
    from mlc_decode_b200 import MlaDecodeKernel
    from mlc_decode_b200.dist import seq_shard

    inputs = O.make_inputs(b, h, s, dt, seed=310 + b)
    ref, rl = _ref(inputs)
    q, qp = inputs[0].to(cuda), inputs[1].to(cuda)
    parts = [seq_shard(s, r, 2) for r in range(2)]
    kvs = [inputs[2][:, a:e].contiguous().to(cuda) for a, e in parts]
    kps = [inputs[3][:, a:e].contiguous().to(cuda) for a, e in parts]
    buf0, buf1 = _buffer(2, b, h, cuda), _buffer(2, b, h, cuda)
    k0 = MlaDecodeKernel(b, h, 1, parts[0][1] - parts[0][0])
    k1 = MlaDecodeKernel(b, h, 1, parts[1][1] - parts[1][0])
    for epoch in (1, 2, 3):
        par = epoch & 1
        # rank 1's contribution, where its launch would have put it: its words in
        # rank 0's buffer, tagged with this call's number
        o1, l1 = _block(buf1, 2, b, h, par, 1)
        k1.partial(q, qp, kvs[1], kps[1], o1, l1)
        _deliver(buf0, 2, b, h, par, 1, o1, l1, epoch)
        torch.cuda.synchronize()
        out = torch.full((b, h, DIM), float("nan"), dtype=q.dtype, device=cuda)
        lse = torch.full((b, h), float("nan"), device=cuda)
        k0.seqsplit(q, qp, kvs[0], kps[0], out, lse, [buf0.data_ptr(), buf1.data_ptr()], 2, 0, epoch)
        torch.cuda.synchronize()
        assert _status(buf0, 2, b, h) == 0
        res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, rl, dt)
        assert res["ok"], (epoch, res)
        # rank 0's rows landed in the peer's words, tagged with this call's number
        o0, l0 = _block(buf0, 2, b, h, par, 0)
        rows, lse_w = _words(buf1, 2, b, h, par, 0)
        assert torch.equal(rows[..., 0], o0.reshape(b * h, DIM).view(torch.int32))
        assert torch.equal(lse_w[:, 0], l0.reshape(b * h).view(torch.int32))
        assert bool((rows[..., 1] == epoch).all()) and bool((lse_w[:, 1] == epoch).all())
        # and they are rank 0's part alone
        r0, rl0 = O.ref_program_f64(inputs[0], inputs[1], inputs[2][:, parts[0][0]:parts[0][1]],
                                    inputs[3][:, parts[0][0]:parts[0][1]])
        assert np.abs(o0.cpu().numpy() - r0).max() < 2e-2
        assert np.abs(l0.cpu().numpy() - rl0).max() < 1e-3


def test_peer_that_never_delivers_times_out(cuda):
    """Nothing from rank 1: the launch gives up (2 s) with status 0x201, and the
    next call on the same context works."""
    from mlc_decode_b200 import MlaDecodeKernel

    b, h, s = 1, 128, 4000
    inputs = O.make_inputs(b, h, s, "bf16", seed=320)
    q, qp, kv, kp = (t.to(cuda) for t in inputs)
    buf0, buf1 = _buffer(2, b, h, cuda), _buffer(2, b, h, cuda)
    k = MlaDecodeKernel(b, h, 1, s)
    out = torch.empty(b, h, DIM, dtype=q.dtype, device=cuda)
    k.seqsplit(q, qp, kv, kp, out, None, [buf0.data_ptr(), buf1.data_ptr()], 2, 0, 1)
    torch.cuda.synchronize()
    assert _status(buf0, 2, b, h) == 0x201
    # the context is usable: a world-1 call on a fresh buffer decodes correctly
    ref, rl = _ref(inputs)
    lse = torch.empty(b, h, device=cuda)
    k.seqsplit(q, qp, kv, kp, out, lse, [_buffer(1, b, h, cuda).data_ptr()], 1, 0, 1)
    torch.cuda.synchronize()
    res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, rl, "bf16")
    assert res["ok"], res


def test_merge_of_written_blocks(cuda):
    """mla_seqsplit_merge alone (the second launch): blocks written by
    mla_decode_partial, one of them an empty part (O = 0, LSE = -inf)."""
    from mlc_decode_b200 import MlaDecodeKernel, capi

    b, h, s = 2, 128, 3000
    inputs = O.make_inputs(b, h, s, "bf16", seed=330)
    ref, rl = _ref(inputs)
    q, qp, kv, kp = (t.to(cuda) for t in inputs)
    buf0, buf1 = _buffer(2, b, h, cuda), _buffer(2, b, h, cuda)
    for epoch in (1, 2):
        par = epoch & 1
        o0, l0 = _block(buf0, 2, b, h, par, 0)
        MlaDecodeKernel(b, h, 1, s).partial(q, qp, kv, kp, o0, l0)
        # rank 1 holds no rows: O = 0, LSE = -inf
        _deliver(buf0, 2, b, h, par, 1, torch.zeros(b, h, DIM, device=cuda),
                 torch.full((b, h), float("-inf"), device=cuda), epoch)
        out = torch.full((b, h, DIM), float("nan"), dtype=torch.float32, device=cuda)
        lse = torch.full((b, h), float("nan"), device=cuda)
        capi.seqsplit_merge([buf0.data_ptr(), buf1.data_ptr()], 2, 0, epoch, b, h, out.data_ptr(), lse.data_ptr(),
                            capi.MLA_DTYPE_F32, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert _status(buf0, 2, b, h) == 0
        res = O.check_parity(out.cpu().numpy(), lse.cpu().numpy(), ref, rl, "fp32")   # float32: no rounding
        assert res["ok"], (epoch, res)
