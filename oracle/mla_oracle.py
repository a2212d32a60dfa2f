"""CPU oracle for absorbed-MLA decode.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it.
The product path (``mlc_decode_b200``) never calls into it and raises when
its CUDA library is missing.

It restates, on the CPU, the algorithm of the reference project
(NiseAzaka/mlc_decode) for the decode hot path:

* ``ref_program_f64`` -- the torch/einops oracle ``ref_program``
  (``baseline_mla.py:167-191``) evaluated exactly in float64 with numpy,
  plus the natural-log log-sum-exp of the same scores.
* ``ref_program_torch`` -- the same sequence of tensor ops in torch on CPU
  tensors of the input dtype (concat, einsum, softmax, einsum), which is what
  the reference runs when handed host tensors.  ``bench.py`` times it as the
  CPU baseline.
* ``split_plan`` -- ``_split_plan`` (``mla_decode.py:9-30``).
* ``splitkv_partials_f64`` / ``combine_f64`` -- the split-KV main kernel's
  per-split partial output and LSE (``mla_decode.py:113-192``) and the LSE
  combine (``mla_decode.py:194-246``), in float64 and natural-log units.
* ``ref_grouped_f64`` / ``ref_multi_token_f64`` -- ``ref_program`` with kv_heads > 1
  and per query position of a multi-token step; ``quantize_e4m3`` /
  ``ref_fp8kv_f64`` -- the FP8 latent cache format and ``ref_program`` over the
  dequantized cache (paths the reference does not have).

Parity is pinned by ``tests/golden/`` fixtures produced by importing the
reference's own ``baseline_mla.ref_program`` and ``mla_decode._split_plan``
(``tests/golden/gen_golden.py``); ``tests/test_oracle.py`` checks this module
against them.
"""
from __future__ import annotations

import math

import numpy as np

DIM = 512      # latent (kv_lora_rank) width, mla_decode.py:36 ``dim``
PE_DIM = 64    # rope width, mla_decode.py:37 ``pe_dim``
SM_SCALE = (DIM + PE_DIM) ** -0.5   # baseline_mla.py:180, mla_decode.py:616


def make_inputs(batch, heads, seqlen_kv, dtype="bf16", seed=0, scale=1.0):
    """Seeded host inputs in the order q, q_pe, kv, k_pe.

    ``torch.Generator().manual_seed(seed)``; ``randn`` in float32, times
    ``scale``, cast to ``dtype``.  Shapes follow the reference prim_func
    signature (``mla_decode.py:66-71``): q[b,h,512], q_pe[b,h,64],
    kv[b,s,1,512], k_pe[b,s,1,64].  ``scale=0.1`` gives the distribution the
    reference's harnesses use (``scripts/check_mla.py:68-71``).
    """
    import torch

    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    g = torch.Generator().manual_seed(int(seed))
    shapes = [(batch, heads, DIM), (batch, heads, PE_DIM),
              (batch, seqlen_kv, 1, DIM), (batch, seqlen_kv, 1, PE_DIM)]
    out = []
    for shp in shapes:
        x = torch.randn(*shp, generator=g, dtype=torch.float32)
        if scale != 1.0:
            x = x * scale
        out.append(x.to(tdt))
    return tuple(out)


def _np64(t):
    import torch

    if isinstance(t, np.ndarray):
        return t.astype(np.float64)
    return t.detach().to(torch.float64).cpu().numpy()


def scores_f64(q, q_pe, kv, k_pe):
    """Raw scores [b, h, s] = [q | q_pe] . [kv | k_pe]^T (baseline_mla.py:185-187)."""
    qf = np.concatenate([_np64(q), _np64(q_pe)], axis=-1)            # [b,h,576]
    kf = np.concatenate([_np64(kv)[:, :, 0, :], _np64(k_pe)[:, :, 0, :]], axis=-1)  # [b,s,576]
    return np.matmul(qf, np.swapaxes(kf, 1, 2))                       # [b,h,s]


def ref_program_f64(q, q_pe, kv, k_pe):
    """Exact oracle: (out[b,h,512] float64, lse[b,h] float64 natural log).

    Follows baseline_mla.py:177-191 with kv_head_num == 1: softmax of the
    concatenated scores divided by sqrt(512+64), then times the latent kv.
    LSE is the natural-log log-sum-exp of the scaled scores.
    """
    s = scores_f64(q, q_pe, kv, k_pe) * SM_SCALE
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    z = e.sum(axis=-1, keepdims=True)
    p = e / z
    v = _np64(kv)[:, :, 0, :]                                         # [b,s,512]
    out = np.matmul(p, v)
    lse = (np.log(z) + m)[..., 0]
    return out, lse


def ref_program_torch(q, q_pe, kv, k_pe):
    """``ref_program`` (baseline_mla.py:167-191) restated with plain torch ops.

    Same op sequence as the reference (head-group rearrange, concat, einsum,
    softmax(scores / sqrt(576)), einsum) in the dtype of its inputs, on
    whatever device they live on; used as the timed CPU baseline.
    """
    import torch

    dim = q.shape[-1]
    pe_dim = q_pe.shape[-1]
    groups = q.shape[1] // kv.shape[2]
    b = q.shape[0]
    qq = q.reshape(b, kv.shape[2], groups, dim).permute(0, 2, 1, 3)       # b g h d
    qp = q_pe.reshape(b, kv.shape[2], groups, pe_dim).permute(0, 2, 1, 3)
    kk = kv.permute(0, 2, 1, 3)                                            # b h s d
    kp = k_pe.permute(0, 2, 1, 3)
    query = torch.cat([qq, qp], dim=-1)
    key = torch.cat([kk, kp], dim=-1)
    scores = torch.einsum("bghd,bhsd->bghs", query, key)
    attn = torch.softmax(scores / ((dim + pe_dim) ** 0.5), dim=-1)
    out = torch.einsum("bghs,bhsd->bghd", attn, kk)
    return out.permute(0, 2, 1, 3).reshape(b, -1, dim)


def make_inputs_ext(batch, q_len, heads, kv_heads, seqlen_kv, dtype="bf16", seed=0, scale=1.0):
    """Seeded host inputs with q_len query positions and kv_heads KV heads:
    q[b,q_len,h,512], q_pe[b,q_len,h,64], kv[b,s,kv_heads,512], k_pe[b,s,kv_heads,64]
    (same generator, draw order and casting as ``make_inputs``)."""
    import torch

    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    g = torch.Generator().manual_seed(int(seed))
    shapes = [(batch, q_len, heads, DIM), (batch, q_len, heads, PE_DIM),
              (batch, seqlen_kv, kv_heads, DIM), (batch, seqlen_kv, kv_heads, PE_DIM)]
    out = []
    for shp in shapes:
        x = torch.randn(*shp, generator=g, dtype=torch.float32)
        if scale != 1.0:
            x = x * scale
        out.append(x.to(tdt))
    return tuple(out)


def ref_grouped_f64(q, q_pe, kv, k_pe):
    """``ref_program`` (baseline_mla.py:177-191) for kv_head_num >= 1, exactly.

    q[b,h,*], kv[b,s,kv_heads,*]: the reference rearranges q as
    "b (h g) d -> b g h d" with g = heads // kv_heads (baseline_mla.py:179-182), so
    query head j reads KV head j // g.  Returns (out[b,h,512], lse[b,h]) in float64.
    """
    kvh = kv.shape[2]
    g = q.shape[1] // kvh
    outs, lses = [], []
    for i in range(kvh):
        o, l = ref_program_f64(q[:, i * g:(i + 1) * g], q_pe[:, i * g:(i + 1) * g], kv[:, :, i:i + 1],
                               k_pe[:, :, i:i + 1])
        outs.append(o)
        lses.append(l)
    return np.concatenate(outs, axis=1), np.concatenate(lses, axis=1)


def ref_multi_token_f64(q, q_pe, kv, k_pe, lens=None):
    """Decode step of q_len query positions per sequence, causal within the step.

    q[b,q_len,h,*], kv[b,s,kv_heads,*], lens[b] KV rows per sequence (None: s).
    Position t of a sequence with L rows attends to its first L - (q_len - 1 - t)
    rows (the step's new tokens are the cache's last q_len rows) with the
    reference's grouped-head scores (``ref_grouped_f64``); a position with no rows
    gives out = 0, lse = -inf.  The reference decodes one position per sequence
    (baseline_mla.py:167-191); this extends it position by position.
    Returns (out[b,q_len,h,512], lse[b,q_len,h]) in float64.
    """
    b, ql, h = q.shape[0], q.shape[1], q.shape[2]
    s = kv.shape[1]
    out = np.zeros((b, ql, h, DIM))
    lse = np.full((b, ql, h), -np.inf)
    for bb in range(b):
        L = s if lens is None else max(0, min(int(lens[bb]), s))
        for t in range(ql):
            n = L - (ql - 1 - t)
            if n <= 0:
                continue
            o, l = ref_grouped_f64(q[bb:bb + 1, t], q_pe[bb:bb + 1, t], kv[bb:bb + 1, :n], k_pe[bb:bb + 1, :n])
            out[bb, t], lse[bb, t] = o[0], l[0]
    return out, lse


def quantize_e4m3(kv, scale):
    """e4m3 (torch.float8_e4m3fn) codes of kv / scale, round to nearest, saturating
    at +-448 (the FP8 latent cache format of mla_decode_fp8kv)."""
    import torch

    x = (kv.float() / float(scale)).clamp(-448.0, 448.0)
    return x.to(torch.float8_e4m3fn)


def ref_fp8kv_f64(q, q_pe, kv_fp8, k_pe, scale):
    """The reference's ``ref_program`` (baseline_mla.py:177-191) over the
    dequantized FP8 cache kv_fp8 * scale, exactly (e4m3 -> float64 is exact).
    The reference has no FP8 path (its notes list FP8 KV as untried,
    docs/mla_decode_best_implementation.md:1693); this is the oracle for one."""
    import torch

    kv = kv_fp8.to(torch.float64) * float(scale)
    return ref_program_f64(q, q_pe, kv, k_pe)


def split_plan(seqlen_kv, num_split, block_n, spread=False):
    """``_split_plan`` (mla_decode.py:9-30): -> (ns, blocks_per_cta, extra).

    nb = ceil(s / block_n) tiles go to ns CTAs.  Even family (spread=False):
    chunk = ceil(s / num_split) rounded up to whole tiles, ns shrinks to
    ceil(nb / blocks_per_cta).  Whole-wave family (spread=True): ns kept
    (clamped to [1, nb]); the first ``extra`` CTAs take one more tile.
    """
    nb = -(-seqlen_kv // block_n)
    if not spread:
        chunk = -(-seqlen_kv // num_split)
        blocks_per_cta = max(1, -(-chunk // block_n))
        ns = max(1, -(-nb // blocks_per_cta))
        return ns, blocks_per_cta, 0
    ns = max(1, min(int(num_split), nb))
    blocks_per_cta, extra = divmod(nb, ns)
    return ns, blocks_per_cta, extra


def split_ranges(seqlen_kv, num_split, block_n, spread=False):
    """Token range [start, end) of every split, as the main kernel walks them.

    mla_decode.py:113-120: split z starts at tile (z*bpc + min(z, extra)) and
    covers bpc (+1 for z < extra) tiles; tokens past seqlen_kv are masked
    (mla_decode.py:123-165), which is the same as clipping the range.
    """
    ns, bpc, extra = split_plan(seqlen_kv, num_split, block_n, spread)
    out = []
    for z in range(ns):
        t0 = (z * bpc + min(z, extra)) * block_n
        nt = bpc + (1 if z < extra else 0)
        t1 = min(seqlen_kv, t0 + nt * block_n)
        out.append((min(t0, seqlen_kv), t1))
    return out


def splitkv_partials_f64(q, q_pe, kv, k_pe, ranges):
    """Per-split normalised partial O and natural-log LSE.

    The split-KV main kernel (mla_decode.py:121-192) computes, for each split
    z over its token range, O_z = softmax_z(S) . V and lse_z; returned as
    (o[ns,b,h,512], lse[ns,b,h]).  An empty range gives O = 0, lse = -inf.
    """
    s = scores_f64(q, q_pe, kv, k_pe) * SM_SCALE
    v = _np64(kv)[:, :, 0, :]
    b, h, _ = s.shape
    o = np.zeros((len(ranges), b, h, DIM))
    lse = np.full((len(ranges), b, h), -np.inf)
    for z, (t0, t1) in enumerate(ranges):
        if t1 <= t0:
            continue
        sz = s[:, :, t0:t1]
        m = sz.max(axis=-1, keepdims=True)
        e = np.exp(sz - m)
        zsum = e.sum(axis=-1, keepdims=True)
        o[z] = np.matmul(e / zsum, v[:, t0:t1])
        lse[z] = (np.log(zsum) + m)[..., 0]
    return o, lse


def combine_f64(o, lse):
    """LSE combine (mla_decode.py:212-246) in natural-log units.

    LSE = log(sum_k exp(lse_k - m)) + m with m = max_k lse_k; splits with
    lse = -inf contribute nothing.  out = sum_k exp(lse_k - LSE) * o_k.
    Inputs are split-major: o[ns,b,h,512], lse[ns,b,h].
    """
    o = np.asarray(o, dtype=np.float64)
    lse = np.asarray(lse, dtype=np.float64)
    m = lse.max(axis=0)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(lse - m_safe[None])
    tot = w.sum(axis=0)
    big = np.log(tot) + m_safe
    scale = np.exp(lse - big[None])
    return (scale[..., None] * o).sum(axis=0), big


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = math.sqrt(float((b * b).sum()))
    return math.sqrt(float(((a - b) ** 2).sum())) / max(den, 1e-300)


def round_to(x, dtype):
    """Round a float64 array to fp16/bf16 (round-to-nearest-even) and back."""
    import torch

    tdt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    return torch.from_numpy(np.asarray(x, dtype=np.float64)).to(tdt).to(torch.float64).numpy()


# Parity gate (north star): max|out - oracle| <= 2e-2 and rel-L2 <= 1e-3 against
# the oracle rounded to the output dtype; |lse - oracle lse| <= 1e-3.
MAX_ABS_TOL = 2e-2
REL_L2_TOL = 1e-3
LSE_TOL = 1e-3


def check_parity(out, lse, oracle_out, oracle_lse, dtype):
    """Return a dict of parity metrics and ``ok`` against the north-star gate."""
    out = np.asarray(out, dtype=np.float64)
    ref_r = round_to(oracle_out, dtype)
    res = {
        "max_abs": float(np.abs(out - oracle_out).max()) if out.size else 0.0,
        "rel_l2": rel_l2(out, ref_r),
        "nan": bool(np.isnan(out).any()),
    }
    if lse is not None:
        res["lse_abs"] = float(np.abs(np.asarray(lse, np.float64) - oracle_lse).max())
    res["ok"] = (not res["nan"] and res["max_abs"] <= MAX_ABS_TOL and res["rel_l2"] <= REL_L2_TOL
                 and res.get("lse_abs", 0.0) <= LSE_TOL)
    return res
