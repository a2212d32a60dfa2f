"""Rows a decode call must not read may hold anything, NaN and Inf included.

A serving KV cache is allocated uninitialised and pages are recycled, so the
rows past a sequence's length (the tail of its last page, or of its contiguous
[max_seqlen] slot), pages no sequence references, and other sequences' rows
can hold non-finite bit patterns.  Softmax weights of masked rows are zero, but
0 x NaN is NaN: the kernels must keep those rows out of P.V entirely.  Every
case fills what must not be read with NaN and +-Inf and checks each sequence
against the float64 oracle over its own rows only.
"""
import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _poison_like(t, gen):
    """NaN, +Inf and -Inf in a seeded pattern, in t's dtype."""
    k = torch.randint(0, 3, t.shape, generator=gen)
    vals = torch.tensor([float("nan"), float("inf"), float("-inf")])
    return vals[k].to(t.dtype)


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


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_contiguous_varlen_tails_nonfinite(dtype, cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    lens = [0, 1, 63, 64, 65, 130, 700, 257, 127, 128]
    b, h, smax = len(lens), 128, 700
    inputs = O.make_inputs(b, h, smax, dtype, seed=191)
    gen = torch.Generator().manual_seed(15)
    kv, kp = inputs[2].clone(), inputs[3].clone()
    for bb, L in enumerate(lens):
        kv[bb, L:] = _poison_like(kv[bb, L:], gen)
        kp[bb, L:] = _poison_like(kp[bb, L:], gen)
    dev = "cuda"
    out = torch.full((b, h, 512), float("nan"), dtype=TDT[dtype], device=dev)
    lse = torch.full((b, h), float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax)
    k(inputs[0].to(dev), inputs[1].to(dev), kv.to(dev), kp.to(dev),
      torch.tensor(lens, dtype=torch.int32, device=dev), out, lse)
    torch.cuda.synchronize()
    _check(out, lse, inputs, lens, dtype)


def _paginate_poisoned(kv, kp, lens, page_size, gen, spare=3):
    """Shuffled pages; every row no sequence owns (tails of last pages, spare pages) poisoned."""
    b = kv.shape[0]
    pages_per = [-(-L // page_size) for L in lens]
    max_pages = max(1, max(pages_per))
    num_pages = sum(pages_per) + spare
    order = torch.randperm(num_pages, generator=gen)
    kv_c = _poison_like(torch.empty(num_pages, page_size, kv.shape[2], 512, dtype=kv.dtype), gen)
    kp_c = _poison_like(torch.empty(num_pages, page_size, kv.shape[2], 64, dtype=kp.dtype), gen)
    table = torch.full((b, max_pages), -1, dtype=torch.int32)
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


@pytest.mark.parametrize("page_size,dtype", [(64, "bf16"), (128, "fp16"), (256, "bf16")])
def test_paged_tails_and_spare_pages_nonfinite(page_size, dtype, cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    lens = [1500, 0, 63, 64, 65, 1, 1000, 333, 4000]
    b, h, smax = len(lens), 128, 4096
    inputs = O.make_inputs(b, h, smax, dtype, seed=192)
    gen = torch.Generator().manual_seed(16)
    kv_c, kp_c, table = _paginate_poisoned(inputs[2], inputs[3], lens, page_size, gen)
    dev = "cuda"
    out = torch.full((b, h, 512), float("nan"), dtype=TDT[dtype], device=dev)
    lse = torch.full((b, h), float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax)
    k(inputs[0].to(dev), inputs[1].to(dev), kv_c.to(dev), kp_c.to(dev),
      torch.tensor(lens, dtype=torch.int32, device=dev), out, lse, block_table=table.to(dev))
    torch.cuda.synchronize()
    _check(out, lse, inputs, lens, dtype)


def test_multi_token_grouped_paged_tails_nonfinite(cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    b, ql, h, kvh, smax, ps = 3, 2, 64, 2, 1024, 64
    lens = [1000, 77, 2]
    q, qp, kv, kp = O.make_inputs_ext(b, ql, h, kvh, smax, "bf16", seed=193)
    ref, ref_lse = O.ref_multi_token_f64(q, qp, kv, kp, lens)
    gen = torch.Generator().manual_seed(17)
    kv_c, kp_c, table = _paginate_poisoned(kv, kp, lens, ps, gen)
    dev = "cuda"
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=dev)
    lse = torch.full(q.shape[:-1], float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax, q_len=ql, kv_heads=kvh)
    k(q.to(dev), qp.to(dev), kv_c.to(dev), kp_c.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev),
      out, lse, block_table=table.to(dev))
    torch.cuda.synchronize()
    o, l = out.float().cpu().numpy(), lse.cpu().numpy()
    for bb in range(b):
        for t in range(ql):
            res = O.check_parity(o[bb, t][None], l[bb, t][None], ref[bb, t][None], ref_lse[bb, t][None], "bf16")
            assert res["ok"], (bb, t, res)


def test_fp8_paged_tails_nonfinite(cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    lens = [700, 5, 129]
    b, h, smax, ps, scale = len(lens), 128, 768, 64, 1 / 16
    q, qp, kv, kp = O.make_inputs(b, h, smax, "bf16", seed=194)
    kv8 = O.quantize_e4m3(kv, scale)
    gen = torch.Generator().manual_seed(18)
    pages_per = [-(-L // ps) for L in lens]
    num_pages = sum(pages_per) + 2
    order = torch.randperm(num_pages, generator=gen)
    kv_c = torch.full((num_pages, ps, 1, 512), 0x7F, dtype=torch.uint8)       # e4m3 NaN codes
    kv_c[..., ::2] = 0xFF
    kp_c = _poison_like(torch.empty(num_pages, ps, 1, 64, dtype=torch.bfloat16), gen)
    table = torch.full((b, max(pages_per)), -1, dtype=torch.int32)
    nxt = 0
    for bb, L in enumerate(lens):
        for i in range(pages_per[bb]):
            pg = int(order[nxt])
            nxt += 1
            table[bb, i] = pg
            r0, r1 = i * ps, min(L, (i + 1) * ps)
            kv_c[pg, :r1 - r0] = kv8[bb, r0:r1].view(torch.uint8)
            kp_c[pg, :r1 - r0] = kp[bb, r0:r1]
    dev = "cuda"
    out = torch.full((b, h, 512), float("nan"), dtype=torch.bfloat16, device=dev)
    lse = torch.full((b, h), float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax)
    k(q.to(dev), qp.to(dev), kv_c.to(dev), kp_c.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev),
      out, lse, block_table=table.to(dev), kv_scale=scale)
    torch.cuda.synchronize()
    o, l = out.float().cpu().numpy(), lse.cpu().numpy()
    for bb, L in enumerate(lens):
        ref, ref_lse = O.ref_fp8kv_f64(q[bb:bb + 1], qp[bb:bb + 1], kv8[bb:bb + 1, :L], kp[bb:bb + 1, :L], scale)
        res = O.check_parity(o[bb:bb + 1], l[bb:bb + 1], ref, ref_lse, "bf16")
        assert res["ok"], (bb, L, res)


@pytest.mark.parametrize("kernel", ["tc", "simt"])
def test_fixed_length_neighbour_rows_nonfinite(kernel, cuda):
    """Fixed-length batch with s not a multiple of the tile: sequence 0's last tile
    spans the first rows of sequence 1.  NaN in sequence 1 gives sequence 1 a NaN
    output (as the reference's own ref_program would) but must not reach sequences 0
    and 2."""
    from mlc_decode_b200 import MlaDecodeKernel

    b, h, s = 3, 128, 777
    q, qp, kv, kp = O.make_inputs(b, h, s, "bf16", seed=195)
    kv, kp = kv.clone(), kp.clone()
    gen = torch.Generator().manual_seed(19)
    kv[1, :200] = _poison_like(kv[1, :200], gen)
    kp[1, :200] = _poison_like(kp[1, :200], gen)
    dev = "cuda"
    out = torch.full((b, h, 512), 0.0, dtype=torch.bfloat16, device=dev)
    lse = torch.full((b, h), 0.0, device=dev)
    MlaDecodeKernel(b, h, 1, s, cfg={"kernel": kernel})(q.to(dev), qp.to(dev), kv.to(dev), kp.to(dev), out, lse)
    torch.cuda.synchronize()
    o, l = out.float().cpu().numpy(), lse.cpu().numpy()
    for bb in (0, 2):
        ref, ref_lse = O.ref_program_f64(q[bb:bb + 1], qp[bb:bb + 1], kv[bb:bb + 1], kp[bb:bb + 1])
        res = O.check_parity(o[bb:bb + 1], l[bb:bb + 1], ref, ref_lse, "bf16")
        assert res["ok"], (bb, res)
