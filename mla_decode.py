"""Drop-in replacement for the reference's ``mla_decode.py`` on B200 (sm_100a).

Same public names, argument order and call contract as NiseAzaka/mlc_decode's
module, so its harnesses (test_mla.py, scripts/check_mla.py,
scripts/bench_mla_heads.py, scripts/tune_best.py, scripts/scan_ns.py,
scripts/mla_prof.py, scripts/dump_kernel_src.py) run unchanged:

* ``_get_kernel(batch, heads, kv_heads, kv_ctx, dim, pe_dim)`` -> kernel
  (mla_decode.py:690-710); ``kernel(q, q_pe, kv, k_pe, out)`` writes ``out``.
* ``run_kernel(q, q_pe, kv, k_pe, output, batch, heads, kv_heads, kv_ctx,
  dim, pe_dim)`` (mla_decode.py:715-717).
* ``build_kernel_from_config(batch, heads, kv_head_num, seqlen_kv, dim,
  pe_dim, cfg)`` (mla_decode.py:720-729).
* ``mla_autotune_configs(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim)``
  (mla_decode.py:539-606), here with B200 candidates.
* ``_split_plan(seqlen_kv, num_split, block_n, spread=False)``
  (mla_decode.py:9-30).
* ``flashattn_shared_q`` / ``flashattn_frag_q`` (mla_decode.py:36-39,
  264-267), positional factory signature; both build the same B200 kernel
  (Q placement is a C500 concern).
* ``flashattn_autotuned`` (mla_decode.py:609-620).

Selection (``_get_kernel``): a tuned entry of ``mla_best_configs_b200.json``
for the shape if there is one, else the library's own heuristic.
``MLA_NO_AUTOTUNE=1`` skips the table (heuristic only), as the reference's
flag skips its autotuner (mla_decode.py:627).  ``MLA_AUTOTUNE=1`` times every
``mla_autotune_configs`` candidate on the first call of a shape and keeps the
fastest.  The kernels run on the current CUDA stream; they need the in-tree
``libmla_decode_b200.so`` and raise if it cannot be loaded.
"""
from __future__ import annotations

import os
import sys

import torch

from mlc_decode_b200 import plan as _plan
from mlc_decode_b200.decode import MlaDecodeKernel

_split_plan = _plan._split_plan
mla_autotune_configs = _plan.mla_autotune_configs

_CACHE_SHARED = {}
_TUNE_CACHE = {}
_AUTOTUNE_ENABLED = os.environ.get("MLA_NO_AUTOTUNE", "0") != "1"
_ONLINE_TUNE = os.environ.get("MLA_AUTOTUNE", "0") == "1"


def _cfg_from_args(block_N, block_H, num_split, num_stages, spread, combine_groups, kernel=None):
    cfg = {"block_N": int(block_N), "block_H": int(block_H), "num_split": int(num_split),
           "num_stages": int(num_stages), "spread": bool(spread),
           "combine_groups": int(combine_groups)}
    if kernel is not None:
        cfg["kernel"] = kernel
    return cfg


def flashattn_shared_q(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, block_N, block_H,
                       num_split, num_stages, dim_chunk_num, softmax_scale, threads=128,
                       spread=False, combine_groups=1, combine_threads=64):
    """Kernel factory with the reference's positional signature (mla_decode.py:36-39).

    block_N / num_split / spread select the KV split exactly as the
    reference's _split_plan does; block_H, num_stages, dim_chunk_num,
    threads, combine_groups and combine_threads are accepted for
    compatibility (the B200 kernels fix their own head grouping and staging).
    """
    cfg = _cfg_from_args(block_N, block_H, num_split, num_stages, spread, combine_groups)
    cfg["kernel"] = _kind_for_block_n(heads, seqlen_kv, block_N)
    return MlaDecodeKernel(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, cfg, softmax_scale)


def flashattn_frag_q(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, block_N, block_H,
                     num_split, num_stages, dim_chunk_num, softmax_scale, threads=128,
                     spread=False, combine_groups=1, combine_threads=64):
    """Same factory as ``flashattn_shared_q`` (mla_decode.py:263-267)."""
    return flashattn_shared_q(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, block_N, block_H,
                              num_split, num_stages, dim_chunk_num, softmax_scale, threads, spread,
                              combine_groups, combine_threads)


def _kind_for_block_n(heads, seqlen_kv, block_n):
    """A reference-style block_N (32/64) means the CUDA-core kernel; 128 the tensor-core one."""
    if int(block_n) % _plan.TC_TILE == 0 and _plan.tc_supported(heads, seqlen_kv):
        return "tc"
    return "simt"


class _AutotunedKernel:
    """Times every candidate on the first call per dtype and keeps the fastest."""

    def __init__(self, batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, warmup=3, rep=10):
        self.args = (batch, heads, kv_head_num, seqlen_kv, dim, pe_dim)
        self.warmup, self.rep = warmup, rep
        self.best = {}
        self.results = {}

    def _tune(self, q, q_pe, kv, k_pe, out):
        rows = []
        for cfg in mla_autotune_configs(*self.args):
            try:
                k = MlaDecodeKernel(*self.args, cfg=cfg)
                for _ in range(self.warmup):
                    k(q, q_pe, kv, k_pe, out)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                for _ in range(self.rep):
                    k(q, q_pe, kv, k_pe, out)
                e.record()
                e.synchronize()
                rows.append((s.elapsed_time(e) * 1000.0 / self.rep, cfg, k))
            except Exception as exc:  # noqa: BLE001 - a config that fails is skipped
                print(f"[mla_decode] config {cfg} failed: {exc}", file=sys.stderr)
        if not rows:
            raise RuntimeError("mla_decode: every autotune candidate failed")
        rows.sort(key=lambda r: r[0])
        self.results[q.dtype] = [(us, cfg) for us, cfg, _ in rows]
        return rows[0][2]

    def __call__(self, q, q_pe, kv, k_pe, out, lse=None):
        k = self.best.get(q.dtype)
        if k is None:
            k = self.best[q.dtype] = self._tune(q, q_pe, kv, k_pe, out)
        k(q, q_pe, kv, k_pe, out, lse)

    def get_kernel_source(self):
        return MlaDecodeKernel(*self.args).get_kernel_source()


def flashattn_autotuned(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, block_N=None,
                        block_H=None, num_split=None, num_stages=None, dim_chunk_num=None,
                        q_in_reg=None, threads=None, spread=None, combine_groups=None):
    """Autotuned build (mla_decode.py:609-620).

    As with the reference's @autotune, passing any tunable argument skips
    tuning and builds that configuration directly.
    """
    tunables = (block_N, num_split, num_stages, spread)
    if any(v is not None for v in tunables):
        cfg = _cfg_from_args(block_N or 0, block_H or 0, num_split or 0, num_stages or 0,
                             spread or False, combine_groups or 1)
        if block_N:
            cfg["kernel"] = _kind_for_block_n(heads, seqlen_kv, block_N)
        return MlaDecodeKernel(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, cfg)
    return _AutotunedKernel(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim)


class _TableKernel:
    """Dispatches per dtype to the tuned table entry, else the library heuristic."""

    def __init__(self, batch, heads, kv_heads, kv_ctx, dim, pe_dim, use_table=True):
        self.args = (batch, heads, kv_heads, kv_ctx, dim, pe_dim)
        self.use_table = use_table
        self.kernels = {}

    def kernel_for(self, dtype):
        k = self.kernels.get(dtype)
        if k is None:
            name = {torch.float16: "fp16", torch.bfloat16: "bf16"}.get(dtype, "other")
            cfg = None
            if self.use_table:
                b, h, _, s, _, _ = self.args
                cfg = _plan.lookup(b, h, s, name)
            k = self.kernels[dtype] = MlaDecodeKernel(*self.args, cfg=cfg)
        return k

    def __call__(self, q, q_pe, kv, k_pe, out, lse=None):
        self.kernel_for(q.dtype)(q, q_pe, kv, k_pe, out, lse)

    def get_kernel_source(self):
        return MlaDecodeKernel(*self.args).get_kernel_source()


def _legacy_kernel(batch, heads, kv_heads, kv_ctx, dim, pe_dim):
    """Heuristic-only kernel (the role of mla_decode.py:630-687)."""
    key = (batch, heads, kv_heads, kv_ctx, dim, pe_dim)
    k = _CACHE_SHARED.get(key)
    if k is None:
        k = _CACHE_SHARED[key] = _TableKernel(*key, use_table=False)
    return k


def _get_kernel(batch, heads, kv_heads, kv_ctx, dim, pe_dim):
    """Kernel for one shape (mla_decode.py:690-710); cached per shape."""
    key = (int(batch), int(heads), int(kv_heads), int(kv_ctx), int(dim), int(pe_dim))
    if not _AUTOTUNE_ENABLED:
        return _legacy_kernel(*key)
    k = _TUNE_CACHE.get(key)
    if k is None:
        k = _AutotunedKernel(*key) if _ONLINE_TUNE else _TableKernel(*key)
        _TUNE_CACHE[key] = k
    return k


def run_kernel(q, q_pe, kv, k_pe, output, batch, heads, kv_heads, kv_ctx, dim, pe_dim):
    """mla_decode.py:715-717."""
    kernel = _get_kernel(int(batch), int(heads), int(kv_heads), int(kv_ctx), int(dim), int(pe_dim))
    kernel(q, q_pe, kv, k_pe, output)


def build_kernel_from_config(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, cfg):
    """Build from an explicit config dict, skipping tuning (mla_decode.py:720-729)."""
    cfg = dict(cfg)
    if "kernel" not in cfg and "block_N" in cfg:
        cfg["kernel"] = _kind_for_block_n(heads, seqlen_kv, cfg["block_N"])
    softmax_scale = (dim + pe_dim) ** -0.5
    return MlaDecodeKernel(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim, cfg, softmax_scale)
