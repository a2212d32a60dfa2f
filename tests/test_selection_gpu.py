"""Kernel selection of the drop-in module on the GPU: the on-line autotuner and the
two environment switches of ``_get_kernel``.

Reference counterparts: ``flashattn_autotuned`` without tunables runs the
autotuner (mla_decode.py:609-620); ``_get_kernel`` uses it unless
``MLA_NO_AUTOTUNE=1`` selects the fixed heuristic (mla_decode.py:627, 690-710).
Here ``MLA_AUTOTUNE=1`` makes ``_get_kernel`` time every candidate on the first
call of a shape, and ``MLA_NO_AUTOTUNE=1`` skips the tuned table.  Each path's
output is checked against the float64 oracle.
"""
import importlib

import pytest
import torch

from oracle import mla_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(2, 16, 1024, "fp16"), (2, 128, 2048, "bf16")]


def _fresh_module(monkeypatch, **env):
    for k in ("MLA_AUTOTUNE", "MLA_NO_AUTOTUNE"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    import mla_decode
    return importlib.reload(mla_decode)


@pytest.fixture(autouse=True)
def _restore_module():
    yield
    import os

    import mla_decode
    saved = {k: os.environ.pop(k) for k in ("MLA_AUTOTUNE", "MLA_NO_AUTOTUNE") if k in os.environ}
    importlib.reload(mla_decode)
    os.environ.update(saved)


def _check(kernel, b, h, s, dt, seed=3):
    cpu = O.make_inputs(b, h, s, dt, seed=seed)
    q, q_pe, kv, k_pe = (t.cuda() for t in cpu)
    out = torch.full_like(q, float("nan"))
    kernel(q, q_pe, kv, k_pe, out)
    torch.cuda.synchronize()
    ref, ref_lse = O.ref_program_f64(*cpu)
    res = O.check_parity(out.float().cpu().numpy(), None, ref, ref_lse, dt)
    assert res["ok"], res
    return out


@pytest.mark.parametrize("b,h,s,dt", SHAPES)
def test_flashattn_autotuned_without_tunables_tunes_online(monkeypatch, cuda, b, h, s, dt):
    m = _fresh_module(monkeypatch)
    k = m.flashattn_autotuned(b, h, 1, s, 512, 64)
    assert isinstance(k, m._AutotunedKernel)
    _check(k, b, h, s, dt)
    tdt = torch.float16 if dt == "fp16" else torch.bfloat16
    rows = k.results[tdt]
    assert len(rows) == len(m.mla_autotune_configs(b, h, 1, s, 512, 64)) > 1
    assert rows[0][0] == min(us for us, _ in rows)   # the fastest candidate is kept
    _check(k, b, h, s, dt, seed=4)                   # later calls reuse it


@pytest.mark.parametrize("b,h,s,dt", SHAPES)
def test_get_kernel_with_MLA_AUTOTUNE_times_candidates(monkeypatch, cuda, b, h, s, dt):
    m = _fresh_module(monkeypatch, MLA_AUTOTUNE="1")
    k = m._get_kernel(b, h, 1, s, 512, 64)
    assert isinstance(k, m._AutotunedKernel)
    assert m._get_kernel(b, h, 1, s, 512, 64) is k   # cached per shape
    _check(k, b, h, s, dt)
    assert k.best


@pytest.mark.parametrize("b,h,s,dt", SHAPES)
def test_get_kernel_with_MLA_NO_AUTOTUNE_uses_the_heuristic(monkeypatch, cuda, b, h, s, dt):
    m = _fresh_module(monkeypatch, MLA_NO_AUTOTUNE="1")
    k = m._get_kernel(b, h, 1, s, 512, 64)
    assert isinstance(k, m._TableKernel) and not k.use_table
    out = _check(k, b, h, s, dt)
    tdt = torch.float16 if dt == "fp16" else torch.bfloat16
    assert k.kernels[tdt].cfg == {}                   # no table entry consulted
    # run_kernel goes through the same selection
    cpu = O.make_inputs(b, h, s, dt, seed=3)
    q, q_pe, kv, k_pe = (t.cuda() for t in cpu)
    out2 = torch.empty_like(q)
    m.run_kernel(q, q_pe, kv, k_pe, out2, b, h, 1, s, 512, 64)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_get_kernel_default_reads_the_tuned_table(monkeypatch, cuda):
    m = _fresh_module(monkeypatch)
    b, h, s, dt = 2, 16, 1024, "fp16"
    k = m._get_kernel(b, h, 1, s, 512, 64)
    assert isinstance(k, m._TableKernel) and k.use_table
    _check(k, b, h, s, dt)
    from mlc_decode_b200 import plan
    ent = plan.lookup(b, h, s, dt)
    if ent is not None:
        assert k.kernels[torch.float16].cfg == ent
