"""GPU parity of mla_decode_ext (query length > 1, grouped KV heads) against the oracle.

Each (sequence, query position) is checked against the float64 oracle
``ref_multi_token_f64`` (position t of a sequence with L KV rows sees its first
L - (q_len - 1 - t) rows; query head j reads KV head j // (heads // kv_heads)).
KV rows past a sequence's length hold large finite garbage, which must be masked.
"""
import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _check(out, lse, ref, ref_lse, dtype):
    out = out.float().cpu().numpy()
    lse = lse.cpu().numpy()
    b, ql = ref.shape[0], ref.shape[1]
    for bb in range(b):
        for t in range(ql):
            if np.all(np.isneginf(ref_lse[bb, t])):
                assert np.all(out[bb, t] == 0.0), (bb, t)
                assert np.all(np.isneginf(lse[bb, t])), (bb, t)
                continue
            res = O.check_parity(out[bb, t][None], lse[bb, t][None], ref[bb, t][None], ref_lse[bb, t][None], dtype)
            assert res["ok"], (bb, t, res)


def _garbage_tails(kv, kp, lens, gen):
    kv, kp = kv.clone(), kp.clone()
    for bb, L in enumerate(lens):
        if L < kv.shape[1]:
            kv[bb, L:] = (torch.rand(kv[bb, L:].shape, generator=gen) * 2000 - 1000).to(kv.dtype)
            kp[bb, L:] = (torch.rand(kp[bb, L:].shape, generator=gen) * 2000 - 1000).to(kp.dtype)
    return kv, kp


def _run(b, ql, h, kvh, smax, lens, dtype, seed, with_lens=True):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    q, qp, kv, kp = O.make_inputs_ext(b, ql, h, kvh, smax, dtype, seed=seed)
    ref, ref_lse = O.ref_multi_token_f64(q, qp, kv, kp, lens if with_lens else None)
    if with_lens:
        kv, kp = _garbage_tails(kv, kp, lens, torch.Generator().manual_seed(seed + 1))
    dev = "cuda"
    if ql == 1:
        q, qp = q[:, 0].contiguous(), qp[:, 0].contiguous()
    out = torch.full(q.shape, float("nan"), dtype=TDT[dtype], device=dev)
    lse = torch.full(q.shape[:-1], float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax, q_len=ql, kv_heads=kvh)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev) if with_lens else None
    k(q.to(dev), qp.to(dev), kv.to(dev), kp.to(dev), sl, out, lse)
    torch.cuda.synchronize()
    assert k.device_status(torch.device(dev), TDT[dtype]) == 0
    if ql == 1:
        out, lse = out[:, None], lse[:, None]
    return out, lse, ref, ref_lse


@pytest.mark.parametrize("h,kvh,dtype", [(128, 2, "bf16"), (128, 4, "fp16"), (64, 8, "bf16"), (256, 2, "bf16"),
                                         (16, 16, "bf16")])
def test_grouped_kv_heads(h, kvh, dtype, cuda):
    lens = [300, 1, 129]
    out, lse, ref, ref_lse = _run(3, 1, h, kvh, 300, lens, dtype, seed=41)
    _check(out, lse, ref, ref_lse, dtype)


@pytest.mark.parametrize("ql,h,dtype", [(2, 128, "bf16"), (3, 64, "fp16"), (4, 16, "bf16"), (2, 200, "bf16")])
def test_multi_token_causal(ql, h, dtype, cuda):
    lens = [700, 1, 2, 129, 128, 0, 3]
    out, lse, ref, ref_lse = _run(len(lens), ql, h, 1, 700, lens, dtype, seed=42)
    _check(out, lse, ref, ref_lse, dtype)


def test_multi_token_grouped_no_lengths(cuda):
    """cache_seqlens None: every sequence holds max_seqlen_kv rows."""
    out, lse, ref, ref_lse = _run(2, 2, 128, 2, 513, [513, 513], "bf16", seed=43, with_lens=False)
    _check(out, lse, ref, ref_lse, "bf16")


def test_multi_token_long_sequence_combine(cuda):
    """One long sequence split over many CTA pairs per position (combine launch)."""
    out, lse, ref, ref_lse = _run(2, 2, 128, 1, 24000, [24000, 100], "bf16", seed=44)
    _check(out, lse, ref, ref_lse, "bf16")


def test_multi_token_grouped_paged(cuda):
    """q_len 2, 2 KV heads, pages of 64 rows in shuffled order."""
    from mlc_decode_b200 import MlaPagedDecodeKernel

    b, ql, h, kvh, smax, ps = 3, 2, 64, 2, 400, 64
    lens = [400, 65, 1]
    q, qp, kv, kp = O.make_inputs_ext(b, ql, h, kvh, smax, "bf16", seed=45)
    ref, ref_lse = O.ref_multi_token_f64(q, qp, kv, kp, lens)
    gen = torch.Generator().manual_seed(46)
    pages_per = [-(-L // ps) for L in lens]
    num_pages = sum(pages_per) + 2
    order = torch.randperm(num_pages, generator=gen)
    kv_c = (torch.rand(num_pages, ps, kvh, 512, generator=gen) * 2000 - 1000).bfloat16()
    kp_c = (torch.rand(num_pages, ps, kvh, 64, generator=gen) * 2000 - 1000).bfloat16()
    table = torch.full((b, max(pages_per)), -1, dtype=torch.int32)
    nxt = 0
    for bb, L in enumerate(lens):
        for i in range(pages_per[bb]):
            pg = int(order[nxt])
            nxt += 1
            table[bb, i] = pg
            r0, r1 = i * ps, min(L, (i + 1) * ps)
            kv_c[pg, :r1 - r0] = kv[bb, r0:r1]
            kp_c[pg, :r1 - r0] = kp[bb, r0:r1]
    dev = "cuda"
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=dev)
    lse = torch.full(q.shape[:-1], float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax, q_len=ql, kv_heads=kvh)
    k(q.to(dev), qp.to(dev), kv_c.to(dev), kp_c.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev), out,
      lse, block_table=table.to(dev))
    torch.cuda.synchronize()
    _check(out, lse, ref, ref_lse, "bf16")


def test_dropin_factory_grouped_kv_heads(cuda):
    """MlaDecodeKernel(batch, heads, kv_head_num > 1, kv_ctx) as the reference factory is called."""
    from mlc_decode_b200 import MlaDecodeKernel

    b, h, kvh, s = 2, 64, 4, 1000
    q, qp, kv, kp = O.make_inputs_ext(b, 1, h, kvh, s, "bf16", seed=47)
    q, qp = q[:, 0].contiguous(), qp[:, 0].contiguous()
    ref, ref_lse = O.ref_grouped_f64(q, qp, kv, kp)
    dev = "cuda"
    out = torch.empty(b, h, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(b, h, device=dev)
    MlaDecodeKernel(b, h, kvh, s)(q.to(dev), qp.to(dev), kv.to(dev), kp.to(dev), out, lse)
    torch.cuda.synchronize()
    res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, ref_lse, "bf16")
    assert res["ok"], res


def test_ext_rejects_bad_grouping(cuda):
    from mlc_decode_b200 import MlaPagedDecodeKernel

    with pytest.raises(ValueError):
        MlaPagedDecodeKernel(2, 100, 256, kv_heads=3)
