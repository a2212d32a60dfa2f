"""Failure detection of the tensor-core kernel on the GPU, without a fault.

Every barrier wait of the decode kernel is bounded; on a timeout the CTA pair
raises its abort flags, records a status code in the workspace and winds down.
mla_selftest_wait_timeout runs that wait code on barriers nothing arrives on:
the waiting CTA must give up after its limit and record the code, its peer must
leave through the abort flag, and the GPU context must stay usable (a decode call
afterwards still matches the oracle).  No reference counterpart: the reference's
kernels have no bounded waits.
"""
import pytest
import torch

from mlc_decode_b200 import capi

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("limit_ms", [5, 50])
def test_wait_times_out_and_reports(limit_ms):
    dev = torch.device("cuda")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    result = torch.zeros(4, dtype=torch.int64, device=dev)
    limit_ns = limit_ms * 1_000_000
    capi.selftest_wait_timeout(status.data_ptr(), result.data_ptr(), limit_ns,
                               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status.item()) == capi.MLA_SELFTEST_STATUS
    gave_up, waited0, left, waited1 = (int(x) for x in result.tolist())
    assert gave_up == 1 and waited0 >= limit_ns           # CTA 0: its own limit ran out
    assert left == 1 and waited1 < 50 * limit_ns          # CTA 1: left via the abort flag, long
    #                                                        before its own 100 x limit


def test_status_untouched_when_nonzero():
    """A status word already holding a code keeps it (the first failure is the one reported)."""
    dev = torch.device("cuda")
    status = torch.full((1,), 0x101, dtype=torch.int32, device=dev)
    result = torch.zeros(4, dtype=torch.int64, device=dev)
    capi.selftest_wait_timeout(status.data_ptr(), result.data_ptr(), 2_000_000,
                               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 0x101


def test_bad_limit_rejected():
    dev = torch.device("cuda")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    result = torch.zeros(4, dtype=torch.int64, device=dev)
    with pytest.raises(capi.MlaError):
        capi.selftest_wait_timeout(status.data_ptr(), result.data_ptr(), 10, 0)
    with pytest.raises(capi.MlaError):
        capi.selftest_wait_timeout(0, result.data_ptr(), 5_000_000, 0)


def test_decode_after_timeouts_matches_oracle():
    """The context survives the self-test: a decode call still agrees with the oracle."""
    from oracle import mla_oracle as orc
    from mlc_decode_b200.decode import MlaDecodeKernel
    dev = torch.device("cuda")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    result = torch.zeros(4, dtype=torch.int64, device=dev)
    capi.selftest_wait_timeout(status.data_ptr(), result.data_ptr(), 5_000_000,
                               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    b, h, s = 2, 128, 1024
    q, qp, kv, kp = orc.make_inputs(b, h, s, "bf16", seed=7)
    k = MlaDecodeKernel(b, h, 1, s)
    out = torch.empty(b, h, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(b, h, dtype=torch.float32, device=dev)
    k(q.to(dev), qp.to(dev), kv.to(dev), kp.to(dev), out, lse)
    torch.cuda.synchronize()
    ref, ref_lse = orc.ref_program_f64(q, qp, kv, kp)
    res = orc.check_parity(out.float().cpu().numpy(), lse.cpu().numpy(), ref, ref_lse, "bf16")
    assert res["ok"], res
