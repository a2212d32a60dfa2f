"""Pin the CPU oracle to the reference's own outputs (tests/golden/)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import mla_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _cases():
    with open(os.path.join(GOLDEN, "ref_program_cases.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "ref_program.npz"))


def _digest(t):
    return hashlib.sha256(t.contiguous().view(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_inputs_regenerate_bit_exact(case):
    """make_inputs reproduces the exact bytes the reference was run on."""
    t = O.make_inputs(case["batch"], case["heads"], case["kv_ctx"], case["dtype"], case["seed"],
                      case["scale"])
    assert [_digest(x) for x in t] == case["sha256"]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_ref_program(case, golden):
    """ref_program_f64 == baseline_mla.ref_program on float64 inputs; LSE too."""
    q, q_pe, kv, k_pe = O.make_inputs(case["batch"], case["heads"], case["kv_ctx"], case["dtype"],
                                      case["seed"], case["scale"])
    out, lse = O.ref_program_f64(q, q_pe, kv, k_pe)
    ref = golden[f"{case['name']}/out64"].astype(np.float64)
    assert np.abs(out - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())
    assert np.abs(lse - golden[f"{case['name']}/lse64"]).max() <= 1e-9


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_torch_restatement_matches_native_reference(case, golden):
    """ref_program_torch in the input dtype reproduces the reference's native-dtype output
    bit for bit, fp16 and bf16, 16 to 128 heads, up to the bench's per-sequence shape
    (bf16 h128 s8192): it is the timed CPU baseline, so it must be the reference's
    arithmetic.  torch's CPU reductions of a long sequence depend on the thread
    count, so each case runs with the thread count its fixture was made with."""
    import torch

    q, q_pe, kv, k_pe = O.make_inputs(case["batch"], case["heads"], case["kv_ctx"], case["dtype"],
                                      case["seed"], case["scale"])
    before = torch.get_num_threads()
    torch.set_num_threads(int(case.get("threads", before)))
    try:
        out = O.ref_program_torch(q, q_pe, kv, k_pe).float().numpy()
    finally:
        torch.set_num_threads(before)
    ref = golden[f"{case['name']}/out_native"]
    np.testing.assert_array_equal(out, ref)


def test_native_reference_is_within_gate_of_exact(golden):
    """Context for the gate: the reference's own bf16/fp16 output vs the exact value."""
    for case in _cases():
        nat = golden[f"{case['name']}/out_native"].astype(np.float64)
        ex = golden[f"{case['name']}/out64"].astype(np.float64)
        assert np.abs(nat - ex).max() < O.MAX_ABS_TOL


def test_split_plan_matches_reference():
    with open(os.path.join(GOLDEN, "split_plan.json")) as f:
        plans = json.load(f)
    assert len(plans) > 1000
    for s, ns, bn, spread, expect in plans:
        assert list(O.split_plan(s, ns, bn, bool(spread))) == expect, (s, ns, bn, spread)


@pytest.mark.parametrize("s,ns,bn,spread", [(3000, 7, 32, False), (3008, 104, 32, True),
                                             (4095, 64, 64, False), (33, 3, 32, True),
                                             (7, 5, 32, False), (131072, 148, 32, True)])
def test_split_ranges_cover_sequence_once(s, ns, bn, spread):
    r = O.split_ranges(s, ns, bn, spread)
    covered = np.zeros(s, dtype=np.int32)
    for t0, t1 in r:
        covered[t0:t1] += 1
    assert (covered == 1).all()


@pytest.mark.parametrize("s,ns,bn,spread", [(1000, 4, 32, False), (1000, 9, 64, True), (33, 2, 32, True)])
def test_splitkv_plus_combine_equals_full(s, ns, bn, spread):
    """The split-KV decomposition (partials + LSE combine) is the full softmax."""
    q, q_pe, kv, k_pe = O.make_inputs(2, 16, s, "fp32", seed=3)
    o, lse = O.splitkv_partials_f64(q, q_pe, kv, k_pe, O.split_ranges(s, ns, bn, spread))
    out, big = O.combine_f64(o, lse)
    ref, ref_lse = O.ref_program_f64(q, q_pe, kv, k_pe)
    assert np.abs(out - ref).max() < 1e-12
    assert np.abs(big - ref_lse).max() < 1e-12


def test_combine_ignores_empty_splits():
    q, q_pe, kv, k_pe = O.make_inputs(1, 16, 64, "fp32", seed=4)
    o, lse = O.splitkv_partials_f64(q, q_pe, kv, k_pe, [(0, 30), (30, 30), (30, 64)])
    assert np.isneginf(lse[1]).all()
    out, _ = O.combine_f64(o, lse)
    ref, _ = O.ref_program_f64(q, q_pe, kv, k_pe)
    assert np.abs(out - ref).max() < 1e-12


def test_parity_gate_catches_planted_error():
    """A mistake planted in the oracle output (one row zeroed) fails the gate."""
    q, q_pe, kv, k_pe = O.make_inputs(1, 16, 128, "bf16", seed=5)
    ref, lse = O.ref_program_f64(q, q_pe, kv, k_pe)
    good = O.round_to(ref, "bf16")
    assert O.check_parity(good, lse, ref, lse, "bf16")["ok"]
    bad = good.copy()
    bad[0, 3] = 0.0
    assert not O.check_parity(bad, lse, ref, lse, "bf16")["ok"]
    assert not O.check_parity(good, lse + 2e-3, ref, lse, "bf16")["ok"]


def _grouped_cases():
    with open(os.path.join(GOLDEN, "ref_program_grouped_cases.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("case", _grouped_cases(), ids=lambda c: c["name"])
def test_grouped_oracle_matches_reference_ref_program(case):
    """ref_grouped_f64 == baseline_mla.ref_program with kv_head_num > 1 (float64 inputs)."""
    golden = np.load(os.path.join(GOLDEN, "ref_program_grouped.npz"))
    q, q_pe, kv, k_pe = O.make_inputs_ext(case["batch"], 1, case["heads"], case["kv_heads"], case["kv_ctx"],
                                          case["dtype"], case["seed"])
    q, q_pe = q[:, 0].contiguous(), q_pe[:, 0].contiguous()
    assert [_digest(x) for x in (q, q_pe, kv, k_pe)] == case["sha256"]
    out, lse = O.ref_grouped_f64(q, q_pe, kv, k_pe)
    ref = golden[f"{case['name']}/out64"].astype(np.float64)
    assert np.abs(out - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())
    # the grouped torch restatement (the CPU baseline) follows the same grouping
    tout = O.ref_program_torch(q.double(), q_pe.double(), kv.double(), k_pe.double()).numpy()
    assert np.abs(tout - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())


def test_multi_token_oracle_follows_the_causal_rule():
    """Position t of a q_len-token step equals the one-token reference on the first
    L - (q_len - 1 - t) rows; q_len = 1 is the plain reference; empty positions are 0 / -inf."""
    b, ql, h, kvh, s = 3, 3, 32, 2, 70
    q, q_pe, kv, k_pe = O.make_inputs_ext(b, ql, h, kvh, s, "bf16", seed=31)
    lens = [70, 2, 40]
    out, lse = O.ref_multi_token_f64(q, q_pe, kv, k_pe, lens)
    for bb, L in enumerate(lens):
        for t in range(ql):
            n = L - (ql - 1 - t)
            if n <= 0:
                assert np.all(out[bb, t] == 0) and np.all(np.isneginf(lse[bb, t]))
                continue
            o, l = O.ref_grouped_f64(q[bb:bb + 1, t], q_pe[bb:bb + 1, t], kv[bb:bb + 1, :n], k_pe[bb:bb + 1, :n])
            np.testing.assert_allclose(out[bb, t], o[0], rtol=0, atol=1e-12)
            np.testing.assert_allclose(lse[bb, t], l[0], rtol=0, atol=1e-12)
    one, one_lse = O.ref_multi_token_f64(q[:, -1:], q_pe[:, -1:], kv, k_pe, None)
    o, l = O.ref_grouped_f64(q[:, -1], q_pe[:, -1], kv, k_pe)
    np.testing.assert_allclose(one[:, 0], o, rtol=0, atol=1e-12)
    np.testing.assert_allclose(one_lse[:, 0], l, rtol=0, atol=1e-12)
