"""GPU parity at the benchmark configurations' own sizes, against the float64 oracle.

The reference checks every context it times against its fp32 torch path
(scripts/check_mla.py:66-83); here every benchmark shape is decoded whole on the
GPU and sampled sequences are compared with the float64 oracle (the oracle on
every sequence of a 2.5 GB call would take minutes on the host):

* long-cache fp16 b132 h128 s16384, the split sweep num_split in {1, 2, 4, 8, 16}
  on both kernels (CUDA-core: KV splits per sequence and the combine launch;
  tensor-core: CTA pairs, sequences split between pairs and merged) plus the
  default plan;
* the head sweep bf16 b128 s4096, h in {16, 32, 64, 128};
* bf16 b512 h128 s4096 on one GPU (the batch-split workload before it is split);
* bf16 b1 h128 s131072, the whole sequence on one GPU (every sequence split
  between all CTA pairs), and the same sequence split in 8 parts and merged
  (the per-GPU work of the 8-GPU sequence split, emulated on one GPU).

Inputs are N(0,1) from a seeded device generator; the sampled sequences are
copied back for the oracle.
"""
import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

TDT = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _inputs(b, h, s, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    t = TDT[dt]
    q = torch.randn(b, h, 512, device="cuda", generator=g).to(t)
    q_pe = torch.randn(b, h, 64, device="cuda", generator=g).to(t)
    kv = torch.empty(b, s, 1, 512, device="cuda", dtype=t)
    k_pe = torch.empty(b, s, 1, 64, device="cuda", dtype=t)
    for i in range(b):   # per sequence: no fp32 copy of the whole cache at once
        kv[i] = torch.randn(s, 1, 512, device="cuda", generator=g).to(t)
        k_pe[i] = torch.randn(s, 1, 64, device="cuda", generator=g).to(t)
    return q, q_pe, kv, k_pe


def _decode(inputs, cfg):
    from mlc_decode_b200 import MlaDecodeKernel

    q, q_pe, kv, k_pe = inputs
    b, h, _ = q.shape
    k = MlaDecodeKernel(b, h, 1, kv.shape[1], cfg=cfg)
    out = torch.full_like(q, float("nan"))
    lse = torch.full((b, h), float("nan"), dtype=torch.float32, device=q.device)
    k(q, q_pe, kv, k_pe, out, lse)
    torch.cuda.synchronize()
    return k, out, lse


def _check_samples(inputs, out, lse, dt, samples):
    q, q_pe, kv, k_pe = inputs
    assert not torch.isnan(out).any()
    for bb in samples:
        sl = slice(bb, bb + 1)
        ref, ref_lse = O.ref_program_f64(q[sl].cpu(), q_pe[sl].cpu(), kv[sl].cpu(), k_pe[sl].cpu())
        res = O.check_parity(out[sl].float().cpu().numpy(), lse[sl].cpu().numpy(), ref, ref_lse, dt)
        assert res["ok"], (bb, res)


@pytest.fixture(scope="module")
def c3_inputs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    x = _inputs(132, 128, 16384, "fp16", seed=31)
    yield x
    del x
    torch.cuda.empty_cache()


@pytest.mark.parametrize("ns", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("kind", ["simt", "tc"])
def test_c3_long_cache_split_sweep(c3_inputs, kind, ns, cuda):
    k, out, lse = _decode(c3_inputs, {"kernel": kind, "num_split": ns})
    plan = k.plan(torch.float16)
    assert plan["kernel"] == kind and plan["splits"] == ns
    _check_samples(c3_inputs, out, lse, "fp16", (0, 77, 131))


def test_c3_long_cache_default_plan(c3_inputs, cuda):
    k, out, lse = _decode(c3_inputs, None)
    assert k.plan(torch.float16)["kernel"] == "tc"
    _check_samples(c3_inputs, out, lse, "fp16", (5, 64, 130))


@pytest.mark.parametrize("h", [16, 32, 64, 128])
def test_c4_head_sweep_at_size(h, cuda):
    x = _inputs(128, h, 4096, "bf16", seed=40 + h)
    _, out, lse = _decode(x, None)
    _check_samples(x, out, lse, "bf16", (0, 63, 127))


def test_c5a_b512_on_one_gpu(cuda):
    x = _inputs(512, 128, 4096, "bf16", seed=51)
    _, out, lse = _decode(x, None)
    _check_samples(x, out, lse, "bf16", (0, 255, 511))


@pytest.fixture(scope="module")
def c5b_inputs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return _inputs(1, 128, 131072, "bf16", seed=52)


def test_c5b_whole_sequence_on_one_gpu(c5b_inputs, cuda):
    k, out, lse = _decode(c5b_inputs, None)
    assert k.plan(torch.bfloat16)["kernel"] == "tc"
    _check_samples(c5b_inputs, out, lse, "bf16", (0,))


def test_c5b_eight_part_sequence_split_emulated(c5b_inputs, cuda):
    """Each of 8 parts (the rows one GPU of the 8-GPU split holds) decoded to a float32
    (O, LSE) by mla_decode_partial, the parts merged by mla_combine."""
    from mlc_decode_b200 import MlaDecodeKernel, combine
    from mlc_decode_b200.dist import seq_shard

    q, q_pe, kv, k_pe = c5b_inputs
    world = 8
    o_all = torch.empty(world, 1, 128, 512, device=cuda)
    l_all = torch.empty(world, 1, 128, device=cuda)
    for r in range(world):
        a, e = seq_shard(kv.shape[1], r, world)
        MlaDecodeKernel(1, 128, 1, e - a).partial(q, q_pe, kv[:, a:e].contiguous(), k_pe[:, a:e].contiguous(),
                                                  o_all[r], l_all[r])
    out = torch.empty_like(q)
    lse = torch.empty(1, 128, device=cuda)
    combine(l_all, o_all, out, lse)
    torch.cuda.synchronize()
    _check_samples(c5b_inputs, out, lse, "bf16", (0,))
