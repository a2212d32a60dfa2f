"""GPU parity: the CUDA decode path (through the C ABI) against the oracle.

Gate (north star): max|out - oracle| <= 2e-2, rel-L2(out, oracle rounded to
the output dtype) <= 1e-3, |lse - oracle lse| <= 1e-3.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _cases():
    with open(os.path.join(GOLDEN, "ref_program_cases.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "ref_program.npz"))


def run_decode(inputs, cfg=None, with_lse=True, device="cuda:0"):
    from mlc_decode_b200 import MlaDecodeKernel

    q, q_pe, kv, k_pe = (t.to(device) for t in inputs)
    b, h, _ = q.shape
    s = kv.shape[1]
    k = MlaDecodeKernel(b, h, 1, s, 512, 64, cfg=cfg)
    out = torch.full_like(q, float("nan"))
    lse = torch.full((b, h), float("nan"), dtype=torch.float32, device=device) if with_lse else None
    k(q, q_pe, kv, k_pe, out, lse)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), (lse.cpu().numpy() if with_lse else None)


KERNEL_CFGS = [
    {"kernel": "simt", "block_N": 32, "num_split": 1},
    {"kernel": "simt", "block_N": 32, "num_split": 7},
    {"kernel": "simt", "block_N": 64, "num_split": 104, "spread": True},
    {},  # library default (AUTO)
]


@pytest.mark.parametrize("cfg", KERNEL_CFGS, ids=lambda c: json.dumps(c, sort_keys=True))
@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_golden_cases(case, cfg, golden, cuda):
    inputs = O.make_inputs(case["batch"], case["heads"], case["kv_ctx"], case["dtype"], case["seed"],
                           case["scale"])
    out, lse = run_decode(inputs, cfg)
    ref = golden[f"{case['name']}/out64"].astype(np.float64)
    ref_lse = golden[f"{case['name']}/lse64"]
    res = O.check_parity(out, lse, ref, ref_lse, case["dtype"])
    assert res["ok"], res
    # also within the gate of the reference's own native-dtype output
    nat = golden[f"{case['name']}/out_native"].astype(np.float64)
    assert np.abs(out - nat).max() <= O.MAX_ABS_TOL


def _tc_ok(h, s):
    from mlc_decode_b200 import plan
    return plan.tc_supported(h, s)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("b,h,s,ns", [(2, 128, 1024, 0), (3, 128, 777, 0), (1, 128, 129, 0),
                                      (2, 128, 4096, 3), (1, 128, 8192, 16), (4, 128, 300, 1),
                                      (1, 128, 1, 0), (2, 128, 127, 0)])
def test_tensor_core_kernel_vs_oracle(b, h, s, ns, dtype, cuda):
    if not _tc_ok(h, s):
        pytest.skip("tensor-core kernel does not cover this shape")
    inputs = O.make_inputs(b, h, s, dtype, seed=100 + s)
    out, lse = run_decode(inputs, {"kernel": "tc", "num_split": ns})
    ref, ref_lse = O.ref_program_f64(*inputs)
    res = O.check_parity(out, lse, ref, ref_lse, dtype)
    assert res["ok"], res


@pytest.mark.parametrize("h", [16, 32, 64, 128])
def test_head_sweep_default_path(h, cuda):
    inputs = O.make_inputs(2, h, 2048, "bf16", seed=h)
    out, lse = run_decode(inputs)
    ref, ref_lse = O.ref_program_f64(*inputs)
    assert O.check_parity(out, lse, ref, ref_lse, "bf16")["ok"]


def test_reference_distribution_x0_1(cuda):
    """randn*0.1 (check_mla.py:68-71) gives near-uniform attention: stresses the sum path."""
    inputs = O.make_inputs(2, 128, 3000, "fp16", seed=0, scale=0.1)
    out, lse = run_decode(inputs)
    ref, ref_lse = O.ref_program_f64(*inputs)
    res = O.check_parity(out, lse, ref, ref_lse, "fp16")
    assert res["ok"], res
    cos = float((out * ref).sum() / np.sqrt((out * out).sum() * (ref * ref).sum()))
    assert cos > 0.99999


@pytest.mark.parametrize("qscale", [3.0, 8.0])
def test_large_scores_stress_the_max_path(qscale, cuda):
    """Scaled-up queries make the softmax peaky (large running-max jumps) while the
    values stay N(0,1), so the max-abs gate keeps its meaning."""
    q, q_pe, kv, k_pe = O.make_inputs(1, 128, 2000, "bf16", seed=9)
    inputs = ((q.float() * qscale).to(q.dtype), (q_pe.float() * qscale).to(q.dtype), kv, k_pe)
    out, lse = run_decode(inputs)
    ref, ref_lse = O.ref_program_f64(*inputs)
    res = O.check_parity(out, lse, ref, ref_lse, "bf16")
    assert res["ok"], res


def test_kernels_agree_at_c2_size_on_sampled_batches(cuda):
    """The DeepSeek-V3-shaped bench case (b64 h128 s8192 bf16): the default path vs the
    CUDA-core path on the full batch, and both vs the oracle on sampled sequences."""
    from mlc_decode_b200 import MlaDecodeKernel

    b, h, s = 64, 128, 8192
    g = torch.Generator(device="cuda").manual_seed(1)
    dev = torch.device("cuda:0")
    q = torch.randn(b, h, 512, device=dev, generator=g).to(torch.bfloat16)
    q_pe = torch.randn(b, h, 64, device=dev, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, s, 1, 512, device=dev, generator=g).to(torch.bfloat16)
    k_pe = torch.randn(b, s, 1, 64, device=dev, generator=g).to(torch.bfloat16)
    outs = []
    for cfg in ({}, {"kernel": "simt"}):
        out = torch.empty_like(q)
        lse = torch.empty(b, h, device=dev)
        MlaDecodeKernel(b, h, 1, s, cfg=cfg)(q, q_pe, kv, k_pe, out, lse)
        outs.append((out.float(), lse))
    torch.cuda.synchronize()
    d = (outs[0][0] - outs[1][0]).abs().max().item()
    assert d <= 2e-2
    for bi in (0, 37, 63):
        ref, ref_lse = O.ref_program_f64(q[bi:bi + 1].cpu(), q_pe[bi:bi + 1].cpu(),
                                         kv[bi:bi + 1].cpu(), k_pe[bi:bi + 1].cpu())
        for out, lse in outs:
            res = O.check_parity(out[bi:bi + 1].cpu().numpy(), lse[bi:bi + 1].cpu().numpy(), ref,
                                 ref_lse, "bf16")
            assert res["ok"], (bi, res)


def test_output_written_on_current_stream(cuda):
    from mlc_decode_b200 import MlaDecodeKernel

    inputs = [t.cuda() for t in O.make_inputs(2, 16, 512, "bf16", seed=11)]
    k = MlaDecodeKernel(2, 16, 1, 512)
    st = torch.cuda.Stream()
    out = torch.zeros_like(inputs[0])
    with torch.cuda.stream(st):
        k(*inputs, out)
    st.synchronize()
    ref, _ = O.ref_program_f64(*[t.cpu() for t in inputs])
    assert np.abs(out.float().cpu().numpy() - ref).max() < 2e-2


def test_drop_in_harness_calls(cuda):
    """The calls the reference's harnesses make (test_mla.py:99-100, check_mla.py:74-75,
    bench_mla_heads.py:134-136, tune_best.py:78-85, scan_ns.py:73-78)."""
    import mla_decode

    b, h, s = 1, 16, 4096
    q, q_pe, kv, k_pe = (t.cuda() for t in O.make_inputs(b, h, s, "fp16", seed=0, scale=0.1))
    ref, _ = O.ref_program_f64(q.cpu(), q_pe.cpu(), kv.cpu(), k_pe.cpu())
    out = torch.empty_like(q)

    mla_decode._get_kernel(b, h, 1, s, 512, 64)(q, q_pe, kv, k_pe, out)
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - ref).max() < 1e-3

    out.zero_()
    mla_decode.run_kernel(q, q_pe, kv, k_pe, out, b, h, 1, s, 512, 64)
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - ref).max() < 1e-3

    scale = (512 + 64) ** -0.5
    kern = mla_decode.flashattn_shared_q(b, h, 1, s, 512, 64, 32, 16, 64, 1, 8, scale, threads=128)
    out.zero_()
    kern(q, q_pe, kv, k_pe, out)
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - ref).max() < 1e-3

    for cfg in mla_decode.mla_autotune_configs(b, h, 1, s, 512, 64):
        out.zero_()
        mla_decode.build_kernel_from_config(b, h, 1, s, 512, 64, cfg)(q, q_pe, kv, k_pe, out)
        torch.cuda.synchronize()
        assert np.abs(out.float().cpu().numpy() - ref).max() < 1e-3, cfg
    assert "mla_" in kern.get_kernel_source()


def test_combine_entry_point_merges_partials(cuda):
    """mla_combine on oracle partials (the cross-GPU merge step) equals the full result."""
    from mlc_decode_b200 import combine

    inputs = O.make_inputs(2, 128, 1000, "bf16", seed=21)
    ranges = [(0, 250), (250, 250), (250, 700), (700, 1000)]
    o, lse = O.splitkv_partials_f64(*inputs, ranges)
    out = torch.empty(2, 128, 512, dtype=torch.bfloat16, device="cuda")
    big = torch.empty(2, 128, dtype=torch.float32, device="cuda")
    combine(torch.from_numpy(lse).float().cuda(), torch.from_numpy(o).float().cuda(), out, big)
    torch.cuda.synchronize()
    ref, ref_lse = O.ref_program_f64(*inputs)
    res = O.check_parity(out.float().cpu().numpy(), big.cpu().numpy(), ref, ref_lse, "bf16")
    assert res["ok"], res


def _f32_check(o, lse, ref, ref_lse):
    """float32 results: no output rounding, so the gate is on the float64 oracle itself."""
    assert not np.isnan(o).any() and not np.isnan(lse).any()
    assert O.rel_l2(o, ref) <= O.REL_L2_TOL, O.rel_l2(o, ref)
    assert np.abs(o - ref).max() <= O.MAX_ABS_TOL
    assert np.abs(lse - ref_lse).max() <= O.LSE_TOL


@pytest.mark.parametrize("cfg", [{}, {"kernel": "simt", "num_split": 1}, {"kernel": "simt", "num_split": 5}],
                         ids=["auto", "simt-ns1", "simt-ns5"])
@pytest.mark.parametrize("b,h,s,dtype", [(2, 128, 1000, "bf16"), (3, 128, 4096, "fp16"), (2, 64, 700, "bf16")])
def test_partial_entry_point_float32(b, h, s, dtype, cfg, cuda):
    """mla_decode_partial: float32 normalised O and LSE of a KV part."""
    from mlc_decode_b200 import MlaDecodeKernel

    inputs = O.make_inputs(b, h, s, dtype, seed=31)
    q, q_pe, kv, k_pe = (t.cuda() for t in inputs)
    k = MlaDecodeKernel(b, h, 1, s, cfg=cfg)
    o = torch.full((b, h, 512), float("nan"), device="cuda")
    lse = torch.full((b, h), float("nan"), device="cuda")
    k.partial(q, q_pe, kv, k_pe, o, lse)
    torch.cuda.synchronize()
    ref, ref_lse = O.ref_program_f64(*inputs)
    _f32_check(o.cpu().numpy(), lse.cpu().numpy(), ref, ref_lse)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_sequence_split_emulated_on_one_gpu(world, cuda):
    """The cross-GPU sequence split, its ranks run one after another on one GPU:
    seq_shard parts -> mla_decode_partial each -> stacked -> mla_combine."""
    from mlc_decode_b200 import MlaDecodeKernel, combine
    from mlc_decode_b200.dist import seq_shard

    b, h, s = 2, 128, 5000
    inputs = O.make_inputs(b, h, s, "bf16", seed=41)
    q, q_pe, kv, k_pe = (t.cuda() for t in inputs)
    o_all = torch.zeros(world, b, h, 512, device="cuda")
    l_all = torch.full((world, b, h), float("-inf"), device="cuda")
    for r in range(world):
        t0, t1 = seq_shard(s, r, world)
        if t1 > t0:
            MlaDecodeKernel(b, h, 1, t1 - t0).partial(q, q_pe, kv[:, t0:t1].contiguous(),
                                                      k_pe[:, t0:t1].contiguous(), o_all[r], l_all[r])
    out = torch.empty(b, h, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(b, h, device="cuda")
    combine(l_all, o_all, out, lse)
    torch.cuda.synchronize()
    ref, ref_lse = O.ref_program_f64(*inputs)
    res = O.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, ref_lse, "bf16")
    assert res["ok"], res


@pytest.mark.parametrize("cfg", [None, {"combine_groups": 2}, {"combine_groups": -1}],
                         ids=["default", "combine_launch", "in_kernel"])
@pytest.mark.parametrize("b,s,dt", [(1, 32768, "bf16"), (2, 20000, "bf16"), (16, 8192, "fp16"), (3, 5000, "bf16")])
def test_many_piece_sequences(b, s, dt, cfg, cuda):
    """Sequences split between many CTA pairs: merged by a second (combine) launch, or,
    with combine_groups < 0, by all of their pairs inside the decode launch (a
    cooperative launch, one launch per call)."""
    from mlc_decode_b200 import MlaDecodeKernel

    in_kernel = cfg is not None and cfg["combine_groups"] < 0
    k = MlaDecodeKernel(b, 128, 1, s, cfg=cfg)
    plan = k.plan(TDT[dt])
    assert plan["kernel"] == "tc" and plan["launches"] == (1 if in_kernel else 2), plan
    inputs = O.make_inputs(b, 128, s, dt, seed=51)
    out, lse = run_decode(inputs, cfg)
    ref, ref_lse = O.ref_program_f64(*inputs)
    res = O.check_parity(out, lse, ref, ref_lse, dt)
    assert res["ok"], res
    # and the float32 variant through the same launches, twice (counters reset)
    q, q_pe, kv, k_pe = (t.cuda() for t in inputs)
    for _ in range(2):
        o = torch.full((b, 128, 512), float("nan"), device="cuda")
        l32 = torch.full((b, 128), float("nan"), device="cuda")
        k.partial(q, q_pe, kv, k_pe, o, l32)
        torch.cuda.synchronize()
        _f32_check(o.cpu().numpy(), l32.cpu().numpy(), ref, ref_lse)
    assert k.device_status(q.device, TDT[dt]) == 0


def test_combine_float32_output(cuda):
    """mla_combine with a float32 out (a result that can be combined again)."""
    from mlc_decode_b200 import combine

    inputs = O.make_inputs(1, 128, 900, "fp16", seed=61)
    o, lse = O.splitkv_partials_f64(*inputs, [(0, 300), (300, 900)])
    out = torch.empty(1, 128, 512, dtype=torch.float32, device="cuda")
    big = torch.empty(1, 128, dtype=torch.float32, device="cuda")
    combine(torch.from_numpy(lse).float().cuda(), torch.from_numpy(o).float().cuda(), out, big)
    torch.cuda.synchronize()
    ref, ref_lse = O.ref_program_f64(*inputs)
    _f32_check(out.cpu().numpy(), big.cpu().numpy(), ref, ref_lse)


@pytest.mark.parametrize("h,dtype", [(16, "bf16"), (48, "fp16"), (100, "bf16"), (200, "bf16"), (256, "fp16")])
def test_tensor_core_kernel_any_head_count(h, dtype, cuda):
    """Head counts other than 128 run on the tensor-core kernel as groups of 128 heads
    (rows past h read as zero and are never stored)."""
    from mlc_decode_b200 import MlaDecodeKernel

    b, s = 3, 1500
    assert MlaDecodeKernel(b, h, 1, s).plan(TDT[dtype])["kernel"] == "tc"
    inputs = O.make_inputs(b, h, s, dtype, seed=81)
    out, lse = run_decode(inputs, {"kernel": "tc"})
    ref, ref_lse = O.ref_program_f64(*inputs)
    res = O.check_parity(out, lse, ref, ref_lse, dtype)
    assert res["ok"], res
