"""mla_decode_fwd_noalloc: the decode call for callers that cannot allocate.

Callers under CUDA-graph capture, servers that forbid allocation on their
serving path, and plugin hosts whose device memory belongs to another runtime
cannot pass a workspace; this entry point takes its split-KV scratch from a
static device array in the library instead.  The test calls it through the C
ABI twice in a row (different inputs each time, so a stale result from the
shared array would show) and compares each result with the regular
workspace-taking entry point, mla_decode_fwd, within the parity tolerance the
other tests use.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from mlc_decode_b200 import capi
from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

B, H, S = 2, 128, 4096
CFG = {"kernel": "simt", "num_split": 8}   # 8 splits: 4.2 MB of scratch, under the 8 MiB array


def _regular(q, q_pe, kv, k_pe, cfg):
    n = capi.workspace_bytes(B, H, S, capi.MLA_DTYPE_BF16, cfg)
    ws = torch.empty(n, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, dtype=torch.float32, device=q.device)
    stream = torch.cuda.current_stream().cuda_stream
    capi.decode_fwd(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(), out.data_ptr(),
                    lse.data_ptr(), ws.data_ptr(), n, B, H, S, capi.MLA_DTYPE_BF16, cfg, stream)
    return out, lse


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    cfg = capi.make_cfg(CFG)
    assert capi.workspace_bytes(B, H, S, capi.MLA_DTYPE_BF16, cfg) <= 8 << 20
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((101, 202)):
        q, q_pe, kv, k_pe = (t.to(cuda) for t in O.make_inputs(B, H, S, "bf16", seed=seed))
        out = torch.full_like(q, float("nan"))
        lse = torch.full((B, H), float("nan"), dtype=torch.float32, device=cuda)
        capi.decode_fwd_noalloc(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(),
                                out.data_ptr(), lse.data_ptr(), B, H, S, capi.MLA_DTYPE_BF16, cfg,
                                stream)
        ref_out, ref_lse = _regular(q, q_pe, kv, k_pe, cfg)
        torch.cuda.synchronize()
        a = out.float().cpu().numpy()
        b = ref_out.float().cpu().numpy()
        assert not np.isnan(a).any(), call
        assert np.abs(a - b).max() <= O.MAX_ABS_TOL, call
        assert O.rel_l2(a, b) <= O.REL_L2_TOL, call
        assert np.abs(lse.cpu().numpy() - ref_lse.cpu().numpy()).max() <= O.LSE_TOL, call


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    cfg = capi.make_cfg({"kernel": "simt", "num_split": 64})   # 64 splits x 256 rows: ~33 MB
    q, q_pe, kv, k_pe = (torch.zeros(*s, dtype=torch.bfloat16, device=cuda)
                         for s in ((B, H, 512), (B, H, 64), (B, S, 1, 512), (B, S, 1, 64)))
    out = torch.zeros_like(q)
    rc = capi.load().mla_decode_fwd_noalloc(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(),
                                            k_pe.data_ptr(), out.data_ptr(), None, B, H, S,
                                            capi.MLA_DTYPE_BF16, ctypes.byref(cfg),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 2
    assert "static array" in capi.last_error()
