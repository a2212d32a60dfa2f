"""Split planning, autotune candidates and the tuned-config table for B200.

The reference derives all of this for a 104-AP MetaX C500 with 64 KB of
shared memory (mla_decode.py:504-606).  The B200 numbers differ: 148 SMs,
up to 227 KB of shared memory per CTA, and two decode kernels (the tcgen05
tensor-core kernel, which takes any head count as groups of 128 heads, and
the CUDA-core kernel, used when a config asks for it).
The config-dict contract is the reference's (mla_decode.py:588-598):
block_N, block_H, num_split, spread, combine_groups, num_stages,
dim_chunk_num, q_in_reg, threads; plus ``kernel`` ("tc"/"simt") here.
Keys the B200 kernels have no use for (dim_chunk_num, q_in_reg, threads,
combine_groups) are accepted and ignored.
"""
from __future__ import annotations

import json
import os

from . import capi

SM_COUNT = 148
DIM, PE_DIM = 512, 64

TABLE_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mla_best_configs_b200.json")

# CUDA-core kernel: 16 heads per CTA, 32-row tiles, two CTAs resident per SM.
SIMT_BLOCK_H = 16
SIMT_TILE = 32
SIMT_CTAS_PER_SM = 2
# Tensor-core kernel: a CTA pair owns a group of (up to) 128 heads of one sequence; 128-row tiles.
TC_HEADS = 128
TC_TILE = 128

_EVEN_CHUNKS = (512, 1024, 2048, 4096)   # KV rows per split, even family
_WAVES = (1, 2, 4)                        # whole-wave family: splits x units ~ waves x slots


def _split_plan(seqlen_kv, num_split, block_n, spread=False):
    """``_split_plan`` (mla_decode.py:9-30) through the C ABI (the kernels' own planner)."""
    return capi.split_plan(seqlen_kv, num_split, block_n, spread)


def tc_supported(heads, seqlen_kv) -> bool:
    """True when the tensor-core kernel covers (heads, seqlen_kv)."""
    cfg = capi.make_cfg({"kernel": "tc"})
    try:
        return capi.workspace_bytes(1, int(heads), int(seqlen_kv), capi.MLA_DTYPE_BF16, cfg) > 0
    except capi.MlaError:
        return False


def mla_autotune_configs(batch, heads, kv_head_num, seqlen_kv, dim, pe_dim):
    """Legal B200 configs for one shape (cf. mla_decode.py:539-606).

    Two split families, as in the reference: the even family (num_split from a
    per-split KV length) and the whole-wave family (num_split chosen so that
    batch x head-groups x num_split fills whole waves of the 148 SMs, with
    spread=True block-level balancing).
    """
    configs = []
    kinds = []
    if tc_supported(heads, seqlen_kv):
        kinds.append(("tc", TC_TILE, -(-heads // TC_HEADS), 1))
    kinds.append(("simt", SIMT_TILE, -(-heads // SIMT_BLOCK_H), SIMT_CTAS_PER_SM))
    for kind, tile, groups, per_sm in kinds:
        nb = -(-seqlen_kv // tile)
        units = batch * groups * (2 if kind == "tc" else 1)  # a tc unit is a CTA pair
        seen = set()
        cands = []
        for chunk in _EVEN_CHUNKS:
            ns = -(-seqlen_kv // chunk)
            cands.append((ns, False))
        for w in _WAVES:
            slots = SM_COUNT * per_sm * w
            ns = max(1, -(-slots // units))
            cands.append((min(ns, nb), True))
        cands.append((1, False))
        for ns, spread in cands:
            eff = _split_plan(seqlen_kv, ns, tile, spread)[0]
            if eff in seen or eff > 4096:
                continue
            seen.add(eff)
            configs.append({"kernel": kind, "block_N": tile,
                            "block_H": TC_HEADS if kind == "tc" else SIMT_BLOCK_H,
                            "num_split": ns, "spread": spread, "combine_groups": 1,
                            "num_stages": 0, "dim_chunk_num": 8, "q_in_reg": False,
                            "threads": 128})
    return configs


def table_key(batch, heads, seqlen_kv, dtype_name, n_gpu=1):
    return f"b{batch}_h{heads}_s{seqlen_kv}_{dtype_name}_g{n_gpu}"


def load_table(path=TABLE_PATH) -> dict:
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        return json.load(f)


def lookup(batch, heads, seqlen_kv, dtype_name, n_gpu=1, path=TABLE_PATH):
    """Tuned config for this shape, or None (keyed by shape, dtype and GPU count)."""
    ent = load_table(path).get(table_key(batch, heads, seqlen_kv, dtype_name, n_gpu))
    if ent is None:
        return None
    return {k: v for k, v in ent.items() if k not in ("latency_us", "default_us")}
