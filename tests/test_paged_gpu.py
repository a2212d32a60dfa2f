"""GPU parity of the ragged / paged decode (mla_decode_paged) against the oracle.

Every sequence is checked against the float64 oracle over its own KV rows;
rows past a sequence's length (the tail of its last page, or of its
contiguous [max_seqlen] slot) hold large finite garbage, which must be masked.
A sequence with no rows must come back as out = 0, lse = -inf.
"""
import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _logical_inputs(b, h, smax, dtype, seed):
    return O.make_inputs(b, h, smax, dtype, seed=seed)


def _check(out, lse, inputs, lens, dtype):
    q, qp, kv, kp = inputs
    out = out.float().cpu().numpy()
    lse = lse.cpu().numpy()
    for bb, L in enumerate(lens):
        if L <= 0:
            assert np.all(out[bb] == 0.0), bb
            assert np.all(np.isneginf(lse[bb])), bb
            continue
        ref, ref_lse = O.ref_program_f64(q[bb:bb + 1], qp[bb:bb + 1], kv[bb:bb + 1, :L], kp[bb:bb + 1, :L])
        res = O.check_parity(out[bb:bb + 1], lse[bb:bb + 1], ref, ref_lse, dtype)
        assert res["ok"], (bb, L, res)


def _garbage_tails(kv, kp, lens, gen):
    kv = kv.clone()
    kp = kp.clone()
    for bb, L in enumerate(lens):
        if L < kv.shape[1]:
            kv[bb, L:] = (torch.rand(kv[bb, L:].shape, generator=gen) * 2000 - 1000).to(kv.dtype)
            kp[bb, L:] = (torch.rand(kp[bb, L:].shape, generator=gen) * 2000 - 1000).to(kp.dtype)
    return kv, kp


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_varlen_contiguous(dtype, cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    b, h, smax = 6, 128, 700
    lens = [0, 1, 130, 700, 64, 257]
    inputs = _logical_inputs(b, h, smax, dtype, seed=91)
    gen = torch.Generator().manual_seed(5)
    kv, kp = _garbage_tails(inputs[2], inputs[3], lens, gen)
    dev = "cuda"
    q, qp = inputs[0].to(dev), inputs[1].to(dev)
    out = torch.full((b, h, 512), float("nan"), dtype=TDT[dtype], device=dev)
    lse = torch.full((b, h), float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax)
    k(q, qp, kv.to(dev), kp.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev), out, lse)
    torch.cuda.synchronize()
    _check(out, lse, inputs, lens, dtype)


def _paginate(kv, kp, lens, page_size, gen, spare=3):
    """Scatter each sequence's rows into shuffled pages; unused rows get garbage."""
    b = kv.shape[0]
    pages_per = [-(-L // page_size) for L in lens]
    max_pages = max(1, max(pages_per))
    num_pages = sum(pages_per) + spare
    order = torch.randperm(num_pages, generator=gen)
    kv_c = (torch.rand(num_pages, page_size, 1, 512, generator=gen) * 2000 - 1000).to(kv.dtype)
    kp_c = (torch.rand(num_pages, page_size, 1, 64, generator=gen) * 2000 - 1000).to(kp.dtype)
    table = torch.full((b, max_pages), -1, dtype=torch.int32)   # entries past a length are never read
    nxt = 0
    for bb, L in enumerate(lens):
        for i in range(pages_per[bb]):
            pg = int(order[nxt])
            nxt += 1
            table[bb, i] = pg
            r0, r1 = i * page_size, min(L, (i + 1) * page_size)
            kv_c[pg, :r1 - r0] = kv[bb, r0:r1]
            kp_c[pg, :r1 - r0] = kp[bb, r0:r1]
    return kv_c, kp_c, table


@pytest.mark.parametrize("page_size,h,dtype", [(64, 128, "bf16"), (128, 64, "bf16"), (256, 128, "fp16")])
def test_paged(page_size, h, dtype, cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    lens = [1500, 0, 63, 64, 65, 1, 1000, 333]
    b, smax = len(lens), 1536
    inputs = _logical_inputs(b, h, smax, dtype, seed=92)
    gen = torch.Generator().manual_seed(6)
    kv_c, kp_c, table = _paginate(inputs[2], inputs[3], lens, page_size, gen)
    dev = "cuda"
    q, qp = inputs[0].to(dev), inputs[1].to(dev)
    out = torch.full((b, h, 512), float("nan"), dtype=TDT[dtype], device=dev)
    lse = torch.full((b, h), float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax)
    k(q, qp, kv_c.to(dev), kp_c.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev), out, lse,
      block_table=table.to(dev))
    torch.cuda.synchronize()
    _check(out, lse, inputs, lens, dtype)


def test_paged_long_sequence_uses_combine(cuda):
    """One long sequence split over many CTA pairs (combine launch) next to short ones
    (merged in the decode kernel), called twice to check the counters reset."""
    from mlc_decode_b200 import MlaPagedDecodeKernel

    lens = [30000, 200, 129, 5]
    b, h, smax, page_size = len(lens), 128, 30016, 64
    inputs = _logical_inputs(b, h, smax, "bf16", seed=93)
    gen = torch.Generator().manual_seed(7)
    kv_c, kp_c, table = _paginate(inputs[2], inputs[3], lens, page_size, gen)
    dev = "cuda"
    q, qp = inputs[0].to(dev), inputs[1].to(dev)
    k = MlaPagedDecodeKernel(b, h, smax)
    seqlens = torch.tensor(lens, dtype=torch.int32, device=dev)
    kv_d, kp_d, tb = kv_c.to(dev), kp_c.to(dev), table.to(dev)
    for _ in range(2):
        out = torch.full((b, h, 512), float("nan"), dtype=torch.bfloat16, device=dev)
        lse = torch.full((b, h), float("nan"), device=dev)
        k(q, qp, kv_d, kp_d, seqlens, out, lse, block_table=tb)
        torch.cuda.synchronize()
        _check(out, lse, inputs, lens, "bf16")
    assert k.device_status(q.device, torch.bfloat16) == 0   # no device-side timeout


def test_paged_rejects_bad_page_size(cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel, capi

    b, h, smax = 2, 128, 256
    dev = "cuda"
    q = torch.zeros(b, h, 512, dtype=torch.bfloat16, device=dev)
    qp = torch.zeros(b, h, 64, dtype=torch.bfloat16, device=dev)
    kv = torch.zeros(8, 96, 1, 512, dtype=torch.bfloat16, device=dev)   # 96-row pages: not a multiple of 64
    kp = torch.zeros(8, 96, 1, 64, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(q)
    table = torch.zeros(b, 3, dtype=torch.int32, device=dev)
    with pytest.raises(capi.MlaError):
        MlaPagedDecodeKernel(b, h, smax)(q, qp, kv, kp, torch.full((b,), 100, dtype=torch.int32, device=dev),
                                         out, block_table=table)
