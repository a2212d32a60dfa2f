"""GPU parity of the FP8 latent KV path (mla_decode_fp8kv) against the oracle.

The cache is quantized on the host (``quantize_e4m3``: kv / scale to e4m3), and
the kernel's output is compared with the float64 reference over the dequantized
cache (``ref_fp8kv_f64``), with the gate of the bf16/fp16 paths: max |err| <= 2e-2,
rel-L2 <= 1e-3 against the oracle rounded to the output dtype, |lse err| <= 1e-3.
"""
import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _run(b, h, s, dtype, seed, scale, x=1.0, cfg=None, calls=1):
    from mlc_decode_b200 import MlaDecodeKernel

    q, qp, kv, kp = O.make_inputs(b, h, s, dtype, seed=seed, scale=x)
    kv8 = O.quantize_e4m3(kv, scale)
    ref, ref_lse = O.ref_fp8kv_f64(q, qp, kv8, kp, scale)
    dev = "cuda"
    k = MlaDecodeKernel(b, h, 1, s, cfg=cfg)
    args = [t.to(dev) for t in (q, qp, kv8, kp)]
    for _ in range(calls):
        out = torch.full((b, h, 512), float("nan"), dtype=TDT[dtype], device=dev)
        lse = torch.full((b, h), float("nan"), device=dev)
        k.decode_fp8(args[0], args[1], args[2], args[3], scale, out, lse)
        torch.cuda.synchronize()
        res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, ref_lse, dtype)
        assert res["ok"], res
    assert k.device_status(torch.device(dev), TDT[dtype]) == 0
    return res


@pytest.mark.parametrize("b,h,s,dtype,scale", [
    (64, 128, 2048, "bf16", 1 / 16),   # whole sequences per CTA pair
    (4, 128, 1000, "bf16", 1 / 16),    # split sequences, merged in the kernel
    (2, 16, 1024, "fp16", 1 / 32),     # the CPU-runnable reference shape, many pieces: combine launch
    (3, 64, 777, "bf16", 0.05),        # rows past h, ragged tail tile, non-power-of-two scale
    (2, 200, 513, "fp16", 1.0),        # two head groups
])
def test_fp8kv_parity(b, h, s, dtype, scale, cuda):
    _run(b, h, s, dtype, seed=61, scale=scale, calls=2)


def test_fp8kv_long_sequence_combine(cuda):
    _run(1, 128, 20000, "bf16", seed=62, scale=1 / 16)


def test_fp8kv_reference_distribution(cuda):
    """The reference harness's randn * 0.1 inputs."""
    _run(2, 128, 4096, "bf16", seed=63, scale=1 / 128, x=0.1)


def test_fp8kv_uint8_bytes_and_errors(cuda):
    """kv given as raw bytes gives the same result; bad scale and the CUDA-core kernel are rejected."""
    from mlc_decode_b200 import MlaDecodeKernel, capi

    b, h, s = 2, 128, 300
    q, qp, kv, kp = O.make_inputs(b, h, s, "bf16", seed=64)
    kv8 = O.quantize_e4m3(kv, 1 / 16)
    dev = "cuda"
    q, qp, kp = q.to(dev), qp.to(dev), kp.to(dev)
    k = MlaDecodeKernel(b, h, 1, s)
    o1 = torch.empty(b, h, 512, dtype=torch.bfloat16, device=dev)
    o2 = torch.empty_like(o1)
    k.decode_fp8(q, qp, kv8.to(dev), kp, 1 / 16, o1)
    k.decode_fp8(q, qp, kv8.view(torch.uint8).to(dev), kp, 1 / 16, o2)
    torch.cuda.synchronize()
    # the same decode (up to the order in which split pieces are merged)
    ref, ref_lse = O.ref_fp8kv_f64(q.cpu(), qp.cpu(), kv8, kp.cpu(), 1 / 16)
    for o in (o1, o2):
        res = O.check_parity(o.float().cpu().numpy(), ref_lse, ref, ref_lse, "bf16")
        assert res["max_abs"] <= 2e-2 and res["rel_l2"] <= 1e-3, res
    with pytest.raises(capi.MlaError):
        k.decode_fp8(q, qp, kv8.to(dev), kp, 0.0, o1)
    with pytest.raises(capi.MlaError):
        MlaDecodeKernel(b, h, 1, s, cfg={"kernel": "simt"}).decode_fp8(q, qp, kv8.to(dev), kp, 1.0, o1)


def test_fp8kv_paged_multi_token_grouped(cuda):
    """The FP8 cache through mla_decode_ext_fp8kv: 64-row pages in shuffled order,
    ragged lengths, q_len 2 (causal within the step) and 2 KV heads."""
    from mlc_decode_b200 import MlaPagedDecodeKernel

    b, ql, h, kvh, smax, ps, scale = 3, 2, 64, 2, 400, 64, 0.05
    lens = [400, 65, 1]
    q, qp, kv, kp = O.make_inputs_ext(b, ql, h, kvh, smax, "bf16", seed=65)
    kv8 = O.quantize_e4m3(kv, scale)
    ref, ref_lse = O.ref_multi_token_f64(q, qp, kv8.to(torch.float64) * scale, kp, lens)
    gen = torch.Generator().manual_seed(66)
    pages_per = [-(-L // ps) for L in lens]
    num_pages = sum(pages_per) + 2
    order = torch.randperm(num_pages, generator=gen)
    kv_c = O.quantize_e4m3(torch.rand(num_pages, ps, kvh, 512, generator=gen) * 400 - 200, 1.0)   # finite garbage
    kp_c = (torch.rand(num_pages, ps, kvh, 64, generator=gen) * 2000 - 1000).bfloat16()
    table = torch.full((b, max(pages_per)), -1, dtype=torch.int32)
    nxt = 0
    for bb, L in enumerate(lens):
        for i in range(pages_per[bb]):
            pg = int(order[nxt])
            nxt += 1
            table[bb, i] = pg
            r0, r1 = i * ps, min(L, (i + 1) * ps)
            kv_c[pg, :r1 - r0] = kv8[bb, r0:r1]
            kp_c[pg, :r1 - r0] = kp[bb, r0:r1]
    dev = "cuda"
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=dev)
    lse = torch.full(q.shape[:-1], float("nan"), device=dev)
    k = MlaPagedDecodeKernel(b, h, smax, q_len=ql, kv_heads=kvh)
    k(q.to(dev), qp.to(dev), kv_c.to(dev), kp_c.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev), out,
      lse, block_table=table.to(dev), kv_scale=scale)
    torch.cuda.synchronize()
    out_n, lse_n = out.float().cpu().numpy(), lse.cpu().numpy()
    for bb in range(b):
        for t in range(ql):
            if np.all(np.isneginf(ref_lse[bb, t])):   # a position with no rows
                assert np.all(out_n[bb, t] == 0.0) and np.all(np.isneginf(lse_n[bb, t])), (bb, t)
                continue
            res = O.check_parity(out_n[bb, t][None], lse_n[bb, t][None], ref[bb, t][None], ref_lse[bb, t][None],
                                 "bf16")
            assert res["ok"], (bb, t, res)
    assert k.device_status(torch.device(dev), torch.bfloat16) == 0
