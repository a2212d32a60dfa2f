"""mla_decode_fwd_noalloc: the decode call for callers that cannot allocate.

Callers under CUDA-graph capture, servers that forbid allocation on their
serving path, and plugin hosts whose device memory belongs to another runtime
cannot pass a workspace; this entry point takes its split-KV scratch from a
static device array in the library instead.  Every case calls it through the
C ABI twice in a row (different inputs each time, so a stale result left in
the shared array would show) and compares each result with the regular
workspace-taking entry point, mla_decode_fwd, and with the float64 oracle on
sampled sequences, within the parity tolerances the other tests use.  The
cases cover both kernels and every way the tensor-core kernel merges a split
sequence (in the kernel by the last of a few pairs or by all pairs of a wide
split, through the status word and piece counters the entry point clears in
the shared array, and in a second combine launch).
This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from mlc_decode_b200 import capi
from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

SCRATCH = 8 << 20

# (name, batch, heads, kv_ctx, cfg, expected tensor-core merge: None = CUDA-core kernel,
#  0 = whole sequences or merged in the kernel (by the last of <= 3 pairs, or by all
#  pairs of a wide split in a cooperative launch), 1 = combine launch)
CASES = [
    ("simt_8_splits", 2, 128, 4096, {"kernel": "simt", "num_split": 8}, None),
    ("tc_whole_sequences", 64, 128, 8192, {"kernel": "tc"}, 0),
    ("tc_merged_in_kernel", 2, 128, 4096, {"kernel": "tc", "num_split": 4}, 0),
    ("tc_merged_by_all_pairs", 1, 128, 32768, {"kernel": "tc", "num_split": 12, "combine_groups": -1}, 0),
    ("tc_combine_launch", 1, 128, 32768, {"kernel": "tc", "num_split": 12}, 1),
]


def _regular(q, q_pe, kv, k_pe, b, h, s, cfg):
    n = capi.workspace_bytes(b, h, s, capi.MLA_DTYPE_BF16, cfg)
    ws = torch.zeros(max(n, 1), dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    lse = torch.empty(b, h, dtype=torch.float32, device=q.device)
    stream = torch.cuda.current_stream().cuda_stream
    capi.decode_fwd(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(), out.data_ptr(),
                    lse.data_ptr(), ws.data_ptr(), n, b, h, s, capi.MLA_DTYPE_BF16, cfg, stream)
    return out, lse


@pytest.mark.parametrize("name,b,h,s,cfg_d,merge", CASES, ids=[c[0] for c in CASES])
def test_noalloc_matches_workspace_entry_point_and_oracle_twice(cuda, name, b, h, s, cfg_d, merge):
    cfg = capi.make_cfg(cfg_d)
    plan = capi.describe_plan(b, h, s, capi.MLA_DTYPE_BF16, cfg)
    assert capi.workspace_bytes(b, h, s, capi.MLA_DTYPE_BF16, cfg) <= SCRATCH
    if merge is None:
        assert plan["kernel"] == "simt"
    else:
        assert plan["kernel"] == "tc"
        assert plan["launches"] == 1 + merge
        assert plan["zero_prefix_bytes"] > 0   # the header the entry point clears each call
    capi.noalloc_init()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(7)
    for call, seed in enumerate((101, 202)):
        cpu = O.make_inputs(b, h, s, "bf16", seed=seed)
        q, q_pe, kv, k_pe = (t.to(cuda) for t in cpu)
        out = torch.full_like(q, float("nan"))
        lse = torch.full((b, h), float("nan"), dtype=torch.float32, device=cuda)
        capi.decode_fwd_noalloc(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(),
                                out.data_ptr(), lse.data_ptr(), b, h, s, capi.MLA_DTYPE_BF16, cfg, stream)
        status = torch.full((1,), 0x7FFFFFFF, dtype=torch.int32, device=cuda)
        capi.noalloc_status(status.data_ptr(), stream)
        ref_out, ref_lse = _regular(q, q_pe, kv, k_pe, b, h, s, cfg)
        torch.cuda.synchronize()
        assert int(status.item()) == 0, (name, call)
        a = out.float().cpu().numpy()
        r = ref_out.float().cpu().numpy()
        assert not np.isnan(a).any(), (name, call)
        assert np.abs(a - r).max() <= O.MAX_ABS_TOL, (name, call)
        assert O.rel_l2(a, r) <= O.REL_L2_TOL, (name, call)
        assert np.abs(lse.cpu().numpy() - ref_lse.cpu().numpy()).max() <= O.LSE_TOL, (name, call)
        # against the float64 oracle on sampled sequences (the first and one other)
        for bb in sorted({0, int(rng.integers(0, b))}):
            o64, l64 = O.ref_program_f64(*(t[bb:bb + 1] for t in cpu))
            res = O.check_parity(a[bb:bb + 1], lse.cpu().numpy()[bb:bb + 1], o64, l64, "bf16")
            assert res["ok"], (name, call, bb, res)


def test_noalloc_status_reads_zero_after_a_call(cuda):
    cfg = capi.make_cfg({"kernel": "tc"})
    b, h, s = 64, 128, 1024   # whole sequences per CTA pair: the workspace is the header only
    q, q_pe, kv, k_pe = (t.to(cuda) for t in O.make_inputs(b, h, s, "bf16", seed=5))
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    capi.decode_fwd_noalloc(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(), out.data_ptr(),
                            None, b, h, s, capi.MLA_DTYPE_BF16, cfg, stream)
    host = torch.full((1,), 0x7FFFFFFF, dtype=torch.int32).pin_memory()
    capi.noalloc_status(host.data_ptr(), stream)
    torch.cuda.synchronize()
    assert int(host.item()) == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    b, h, s = 2, 128, 4096
    cfg = capi.make_cfg({"kernel": "simt", "num_split": 64})   # 64 splits x 256 rows: ~33 MB
    q, q_pe, kv, k_pe = (torch.zeros(*sh, dtype=torch.bfloat16, device=cuda)
                         for sh in ((b, h, 512), (b, h, 64), (b, s, 1, 512), (b, s, 1, 64)))
    out = torch.zeros_like(q)
    rc = capi.load().mla_decode_fwd_noalloc(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(),
                                            k_pe.data_ptr(), out.data_ptr(), None, b, h, s,
                                            capi.MLA_DTYPE_BF16, ctypes.byref(cfg),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert "static array" in capi.last_error()


def test_noalloc_rejected_call_enqueues_nothing(cuda):
    """A null input is refused before the shared array's header is touched."""
    b, h, s = 2, 128, 1024
    cfg = capi.make_cfg({"kernel": "tc"})
    out = torch.zeros(b, h, 512, dtype=torch.bfloat16, device=cuda)
    rc = capi.load().mla_decode_fwd_noalloc(None, out.data_ptr(), out.data_ptr(), out.data_ptr(),
                                            out.data_ptr(), None, b, h, s, capi.MLA_DTYPE_BF16,
                                            ctypes.byref(cfg), torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert "null" in capi.last_error()
