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
    (2, 16, 1024, "fp16", 1 / 32),     # BASELINE configs[0] shape, many pieces: combine launch
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
    assert torch.equal(o1, o2)
    with pytest.raises(capi.MlaError):
        k.decode_fp8(q, qp, kv8.to(dev), kp, 0.0, o1)
    with pytest.raises(capi.MlaError):
        MlaDecodeKernel(b, h, 1, s, cfg={"kernel": "simt"}).decode_fp8(q, qp, kv8.to(dev), kp, 1.0, o1)
