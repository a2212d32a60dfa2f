"""Host side of the decode path: the callable kernel object and its workspace.

``MlaDecodeKernel`` is what the reference's ``_get_kernel`` /
``flashattn_shared_q`` return (a TileLang ``JITKernel`` there,
mla_decode.py:690-710): ``kernel(q, q_pe, kv, k_pe, out)`` writes ``out`` in
place on the current CUDA stream.  The reference allocates its ``glse`` /
``output_partial`` scratch inside the kernel on every call
(mla_decode.py:73-76); here the object owns a workspace per (device, dtype),
allocated on first use and reused, and passes it through the C ABI.
"""
from __future__ import annotations

import os
import threading

import torch

from . import capi

DIM = 512
PE_DIM = 64
_DTYPES = {torch.float16: capi.MLA_DTYPE_F16, torch.bfloat16: capi.MLA_DTYPE_BF16}
_FP8 = getattr(torch, "float8_e4m3fn", torch.uint8)


def _check_tensor(name, t, shape, dtype, device):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} has dtype {t.dtype}, expected {dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


class MlaDecodeKernel:
    """Absorbed-MLA decode for one (batch, heads, kv_heads, kv_ctx, dim, pe_dim).

    ``cfg`` is a reference-style config dict (keys block_N, block_H, num_split,
    spread, num_stages, combine_groups; plus ``kernel`` = "auto"/"simt"/"tc"),
    or None to let the library choose.  dim == 512 and pe_dim == 64.  The
    reference's kernels take kv_heads == 1 only (baseline_mla.py:16); here
    kv_head_num > 1 (heads a multiple of it, kv [batch, kv_ctx, kv_head_num,
    512]) runs through mla_decode_ext with the reference ref_program's head
    grouping, for ``__call__`` only.
    """

    def __init__(self, batch, heads, kv_head_num, seqlen_kv, dim=DIM, pe_dim=PE_DIM, cfg=None,
                 softmax_scale=None):
        kvh = int(kv_head_num)
        if kvh < 1 or int(heads) % kvh != 0:
            raise ValueError(f"kv_head_num must be >= 1 and divide heads, got {kv_head_num} for {heads} heads")
        self._grouped = None
        if kvh > 1:
            if (cfg or {}).get("kernel", "auto") == "simt":
                raise ValueError("kv_head_num > 1 runs on the tensor-core kernel only")
            self._grouped = MlaPagedDecodeKernel(batch, heads, seqlen_kv, cfg=cfg, softmax_scale=softmax_scale,
                                                 kv_heads=kvh)
        if int(dim) != DIM or int(pe_dim) != PE_DIM:
            raise ValueError(f"dim/pe_dim must be {DIM}/{PE_DIM}, got {dim}/{pe_dim}")
        if int(batch) < 1 or int(heads) < 1 or int(seqlen_kv) < 1:
            raise ValueError("batch, heads and seqlen_kv must be >= 1")
        self.batch, self.heads, self.seqlen_kv = int(batch), int(heads), int(seqlen_kv)
        self.kv_heads, self.dim, self.pe_dim = kvh, DIM, PE_DIM
        self.cfg = dict(cfg or {})
        if softmax_scale is not None:
            self.cfg["softmax_scale"] = float(softmax_scale)
        self._ccfg = capi.make_cfg(self.cfg)
        capi.load()   # fail loudly now if the library is unusable
        self._ws = {}
        self._lock = threading.Lock()
        b, h, s = self.batch, self.heads, self.seqlen_kv
        self._shapes = (torch.Size((b, h, DIM)), torch.Size((b, h, PE_DIM)), torch.Size((b, s, 1, DIM)),
                        torch.Size((b, s, 1, PE_DIM)))

    # -- workspace ---------------------------------------------------------
    def workspace_bytes(self, dtype: torch.dtype) -> int:
        if self._grouped is not None:
            return self._grouped.workspace_bytes(dtype)
        return capi.workspace_bytes(self.batch, self.heads, self.seqlen_kv, _DTYPES[dtype], self._ccfg)

    def _one_kv_head(self, what):
        if self._grouped is not None:
            raise NotImplementedError(f"{what} takes kv_head_num == 1 (this kernel has {self.kv_heads})")

    def _workspace(self, device, dtype):
        key = (device.index, dtype)
        ws = self._ws.get(key)
        if ws is None:
            with self._lock:
                ws = self._ws.get(key)
                if ws is None:
                    n = self.workspace_bytes(dtype)
                    # zeroed once: the first word is the kernels' status word
                    ws = torch.zeros(max(n, 1), dtype=torch.uint8, device=device)
                    self._ws[key] = ws
        return ws

    # -- call ----------------------------------------------------------------
    def __call__(self, q, q_pe, kv, k_pe, out, lse=None):
        """Write softmax(([q|q_pe].[kv|k_pe]^T) * scale) . kv into ``out``.

        ``lse`` (optional, float32 [batch, heads]) receives the natural-log
        log-sum-exp of the scaled scores.
        """
        if self._grouped is not None:
            self._grouped(q, q_pe, kv, k_pe, None, out, lse)
            return
        b, h, s = self.batch, self.heads, self.seqlen_kv
        dtype = q.dtype if isinstance(q, torch.Tensor) else None
        if dtype not in _DTYPES:
            raise ValueError(f"q must be float16 or bfloat16, got {dtype}")
        dev = q.device
        shapes = self._shapes
        # one pass over the tensors; the detailed checker only runs to explain a failure
        for name, t, shape in (("q", q, shapes[0]), ("q_pe", q_pe, shapes[1]), ("kv", kv, shapes[2]),
                               ("k_pe", k_pe, shapes[3]), ("out", out, shapes[0])):
            if not (type(t) is torch.Tensor and t.dtype == dtype and t.device == dev and t.shape == shape
                    and t.is_contiguous() and dev.type == "cuda"):
                _check_tensor(name, t, shape, dtype, dev)
        lse_ptr = None
        if lse is not None:
            _check_tensor("lse", lse, (b, h), torch.float32, dev)
            lse_ptr = lse.data_ptr()
        ws = self._workspace(dev, dtype)
        stream = torch.cuda.current_stream(dev).cuda_stream
        capi.decode_fwd(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(), out.data_ptr(),
                        lse_ptr, ws.data_ptr(), ws.numel(), b, h, s, _DTYPES[dtype], self._ccfg, stream)

    def decode_fp8(self, q, q_pe, kv_fp8, k_pe, kv_scale, out, lse=None):
        """``__call__`` over an FP8 latent cache (mla_decode_fp8kv).

        ``kv_fp8`` [batch, kv_ctx, 1, 512] holds e4m3 values (``torch.float8_e4m3fn``,
        or their bytes as ``torch.uint8``); the latent rows are ``kv_fp8 * kv_scale``.
        q, q_pe, k_pe and out keep the model dtype.  Tensor-core kernel only.
        """
        self._one_kv_head("decode_fp8")
        b, h, s = self.batch, self.heads, self.seqlen_kv
        dtype = q.dtype if isinstance(q, torch.Tensor) else None
        if dtype not in _DTYPES:
            raise ValueError(f"q must be float16 or bfloat16, got {dtype}")
        if not isinstance(kv_fp8, torch.Tensor) or kv_fp8.dtype not in (torch.uint8, _FP8):
            raise ValueError("kv_fp8 must be a torch.float8_e4m3fn (or uint8) tensor")
        dev = q.device
        _check_tensor("q", q, (b, h, DIM), dtype, None)
        _check_tensor("q_pe", q_pe, (b, h, PE_DIM), dtype, dev)
        _check_tensor("kv_fp8", kv_fp8, (b, s, 1, DIM), kv_fp8.dtype, dev)
        _check_tensor("k_pe", k_pe, (b, s, 1, PE_DIM), dtype, dev)
        _check_tensor("out", out, (b, h, DIM), dtype, dev)
        lse_ptr = None
        if lse is not None:
            _check_tensor("lse", lse, (b, h), torch.float32, dev)
            lse_ptr = lse.data_ptr()
        ws = self._workspace(dev, dtype)
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
        capi.decode_fp8kv(q.data_ptr(), q_pe.data_ptr(), kv_fp8.data_ptr(), k_pe.data_ptr(), float(kv_scale),
                          out.data_ptr(), lse_ptr, ws.data_ptr(), ws.numel(), b, h, s, _DTYPES[dtype], self._ccfg,
                          stream)

    def partial(self, q, q_pe, kv, k_pe, o, lse):
        """Decode against this KV part with a float32 result (mla_decode_partial).

        ``o`` float32 [batch, heads, 512] receives the normalised output and
        ``lse`` float32 [batch, heads] the natural-log log-sum-exp; results of
        several parts of the same sequences merge with :func:`combine`.
        """
        self._one_kv_head("partial")
        b, h, s = self.batch, self.heads, self.seqlen_kv
        dtype = q.dtype if isinstance(q, torch.Tensor) else None
        if dtype not in _DTYPES:
            raise ValueError(f"q must be float16 or bfloat16, got {dtype}")
        dev = q.device
        shapes = self._shapes
        for name, t, shape, dt in (("q", q, shapes[0], dtype), ("q_pe", q_pe, shapes[1], dtype),
                                   ("kv", kv, shapes[2], dtype), ("k_pe", k_pe, shapes[3], dtype),
                                   ("o", o, shapes[0], torch.float32), ("lse", lse, shapes[0][:2], torch.float32)):
            if not (type(t) is torch.Tensor and t.dtype == dt and t.device == dev and t.shape == shape
                    and t.is_contiguous() and dev.type == "cuda"):
                _check_tensor(name, t, shape, dt, dev)
        ws = self._workspace(dev, dtype)
        stream = torch.cuda.current_stream(dev).cuda_stream
        capi.decode_partial(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(), o.data_ptr(),
                            lse.data_ptr(), ws.data_ptr(), ws.numel(), b, h, s, _DTYPES[dtype],
                            self._ccfg, stream)

    def seqsplit(self, q, q_pe, kv, k_pe, out, lse, bufs, world: int, rank: int, epoch: int):
        """This KV part of a sequence split across ranks, and the exchange and merge
        with the other ranks' parts in one more launch (mla_seqsplit_decode): ``out``
        ([batch, heads, 512], q's dtype) and ``lse`` (float32 or None) receive the
        decode over every rank's rows.  ``bufs``: every rank's gather buffer (device
        pointers, a ctypes c_void_p array or a sequence); ``epoch``: this call's
        number, from 1, the same on every rank.  Every rank must call it.
        """
        self._one_kv_head("seqsplit")
        b, h, s = self.batch, self.heads, self.seqlen_kv
        dtype = q.dtype if isinstance(q, torch.Tensor) else None
        if dtype not in _DTYPES:
            raise ValueError(f"q must be float16 or bfloat16, got {dtype}")
        dev = q.device
        shapes = self._shapes
        checks = [("q", q, shapes[0], dtype), ("q_pe", q_pe, shapes[1], dtype), ("kv", kv, shapes[2], dtype),
                  ("k_pe", k_pe, shapes[3], dtype), ("out", out, shapes[0], dtype)]
        if lse is not None:
            checks.append(("lse", lse, shapes[0][:2], torch.float32))
        for name, t, shape, dt in checks:
            if not (type(t) is torch.Tensor and t.dtype == dt and t.device == dev and t.shape == shape
                    and t.is_contiguous() and dev.type == "cuda"):
                _check_tensor(name, t, shape, dt, dev)
        ws = self._workspace(dev, dtype)
        stream = torch.cuda.current_stream(dev).cuda_stream
        capi.seqsplit_decode(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(), out.data_ptr(),
                             None if lse is None else lse.data_ptr(), ws.data_ptr(), ws.numel(), b, h, s,
                             _DTYPES[dtype], bufs, world, rank, epoch, self._ccfg, stream)

    def splitkv(self, q, q_pe, kv, k_pe, out, lse=None):
        """First launch of a call only (the split-KV kernel); pair with ``combine_ws``.

        Device pointers and shapes are trusted to match a previous checked call.
        """
        self._one_kv_head("splitkv")
        ws = self._workspace(q.device, q.dtype)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        capi.decode_splitkv(q.data_ptr(), q_pe.data_ptr(), kv.data_ptr(), k_pe.data_ptr(), out.data_ptr(),
                            None if lse is None else lse.data_ptr(), ws.data_ptr(), ws.numel(),
                            self.batch, self.heads, self.seqlen_kv, _DTYPES[q.dtype], self._ccfg, stream)

    def combine_ws(self, out, lse=None):
        """Second launch of a call: combine the partials ``splitkv`` left in the workspace."""
        self._one_kv_head("combine_ws")
        ws = self._workspace(out.device, out.dtype)
        stream = torch.cuda.current_stream(out.device).cuda_stream
        capi.decode_combine_ws(out.data_ptr(), None if lse is None else lse.data_ptr(), ws.data_ptr(),
                               ws.numel(), self.batch, self.heads, self.seqlen_kv, _DTYPES[out.dtype],
                               self._ccfg, stream)

    def device_status(self, device, dtype) -> int:
        """Status word the tensor-core kernel leaves in the workspace (0 = no timeout)."""
        if self._grouped is not None:
            return self._grouped.device_status(device, dtype)
        ws = self._ws.get((torch.device(device).index, dtype))
        if ws is None or ws.numel() < 4:
            return 0
        return int(ws[:4].view(torch.int32).item())

    def clock_probe(self, device, dtype) -> tuple:
        """(SM cycles, ns, calls) the tensor-core kernel has accumulated in this
        workspace: one CTA's run per call, timed by clock64 and %globaltimer, so
        cycles / ns is the SM clock (GHz) while the kernel ran.  Reads the device
        (synchronises the stream)."""
        return _clock_probe(self._grouped._ws if self._grouped is not None else self._ws, device, dtype)

    def plan(self, dtype=torch.bfloat16) -> dict:
        """The library's plan for this shape: kernel, splits/pairs, launches per call."""
        self._one_kv_head("plan")
        return capi.describe_plan(self.batch, self.heads, self.seqlen_kv, _DTYPES[dtype], self._ccfg)

    def launches_per_call(self, dtype=torch.bfloat16) -> int:
        """Kernels one call enqueues."""
        return self.plan(dtype)["launches"]

    def get_kernel_source(self) -> str:
        """CUDA source of the kernels this object launches (cf. dump_kernel_src.py:40)."""
        here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "csrc")
        parts = []
        for name in ("mla_sm100.cu", "mla_simt.cu", "mla_combine.cu"):
            with open(os.path.join(here, name)) as f:
                parts.append(f"// ===== {name} =====\n" + f.read())
        return "\n".join(parts)

    def __repr__(self):
        return (f"MlaDecodeKernel(batch={self.batch}, heads={self.heads}, seqlen_kv={self.seqlen_kv}, "
                f"cfg={self.cfg})")


def _clock_probe(ws_map, device, dtype):
    ws = ws_map.get((torch.device(device).index, dtype))
    if ws is None or ws.numel() < 32:
        return (0, 0, 0)
    v = ws[8:32].view(torch.int64).tolist()
    return (int(v[0]), int(v[1]), int(v[2]))


def _split_major_view(name, t, inner_shape, device):
    """Checks a [ns, *inner_shape] float32 view whose split dimension may have any
    stride while each split is contiguous; returns the split stride in elements."""
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda" or t.dtype != torch.float32:
        raise ValueError(f"{name} must be a float32 CUDA tensor")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if tuple(t.shape[1:]) != tuple(inner_shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected (ns, {', '.join(map(str, inner_shape))})")
    inner = 1
    for d in range(t.dim() - 1, 0, -1):
        if t.shape[d] != 1 and t.stride(d) != inner:
            raise ValueError(f"{name}: every split must be contiguous")
        inner *= t.shape[d]
    return t.stride(0) if t.shape[0] > 1 else inner


def combine(part_lse: torch.Tensor, part_o: torch.Tensor, out: torch.Tensor, lse=None):
    """LSE-merge ``num_split`` normalised partials into ``out``.

    part_lse float32 [ns, b, h] (natural log), part_o float32 [ns, b, h, 512]:
    split-major, or views whose split dimension has any stride (each split
    contiguous, e.g. the per-GPU blocks of one packed all-gather buffer).
    ``out`` is float16, bfloat16 or float32 [b, h, 512].
    """
    ns, b, h = part_lse.shape
    dev = part_lse.device
    lse_stride = _split_major_view("part_lse", part_lse, (b, h), None)
    o_stride = _split_major_view("part_o", part_o, (b, h, DIM), dev)
    out_types = dict(_DTYPES)
    out_types[torch.float32] = capi.MLA_DTYPE_F32
    if out.dtype not in out_types:
        raise ValueError("out must be float16, bfloat16 or float32")
    _check_tensor("out", out, (b, h, DIM), out.dtype, dev)
    lse_ptr = None
    if lse is not None:
        _check_tensor("lse", lse, (b, h), torch.float32, dev)
        lse_ptr = lse.data_ptr()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
    if part_lse.is_contiguous() and part_o.is_contiguous():
        capi.combine(part_lse.data_ptr(), part_o.data_ptr(), ns, b, h, out.data_ptr(), lse_ptr,
                     out_types[out.dtype], stream)
    else:
        capi.combine_strided(part_lse.data_ptr(), lse_stride, part_o.data_ptr(), o_stride, ns, b, h,
                             out.data_ptr(), lse_ptr, out_types[out.dtype], stream)


class MlaPagedDecodeKernel:
    """Decode over KV caches of different lengths, optionally paged, with
    ``q_len`` query positions per sequence and ``kv_heads`` KV heads.

    ``kernel(q, q_pe, kv_cache, k_pe_cache, cache_seqlens, out, lse=None,
    block_table=None)``: ``cache_seqlens`` int32 [batch] gives each sequence's
    KV rows (at most ``max_seqlen_kv``), or None for all ``max_seqlen_kv``.
    Without ``block_table`` the caches are [batch, max_seqlen_kv, kv_heads, 512]
    / [..., 64]; with it (int32 [batch, max_pages]) they are pages [num_pages,
    page_size, kv_heads, 512] / [..., 64] and row r of sequence b is row r %
    page_size of page block_table[b, r // page_size].  page_size is a multiple
    of 64.  q / out are [batch, heads, 512] for q_len == 1, else [batch, q_len,
    heads, 512] (lse [batch, heads] / [batch, q_len, heads]); position t of a
    sequence of L rows sees its first L - (q_len - 1 - t) rows.  Query head j
    reads KV head j // (heads // kv_heads), as the reference's ref_program
    groups them (baseline_mla.py:179-186).  No counterpart in the reference
    (one kv_ctx, one query position and kv_heads == 1 per call there); the C
    entry points are mla_decode_paged and mla_decode_ext.
    """

    def __init__(self, batch, heads, max_seqlen_kv, cfg=None, softmax_scale=None, q_len=1, kv_heads=1):
        self.batch, self.heads, self.max_seqlen_kv = int(batch), int(heads), int(max_seqlen_kv)
        self.q_len, self.kv_heads = int(q_len), int(kv_heads)
        if self.q_len < 1 or self.kv_heads < 1 or self.heads % self.kv_heads != 0:
            raise ValueError(f"q_len and kv_heads must be >= 1 and divide heads (q_len {q_len}, heads {heads}, "
                             f"kv_heads {kv_heads})")
        self.cfg = dict(cfg or {})
        if softmax_scale is not None:
            self.cfg["softmax_scale"] = float(softmax_scale)
        self._ccfg = capi.make_cfg(self.cfg)
        capi.load()
        self._ws = {}
        self._lock = threading.Lock()

    def workspace_bytes(self, dtype: torch.dtype) -> int:
        return capi.ext_workspace_bytes(self.batch, self.q_len, self.heads, self.kv_heads, self.max_seqlen_kv,
                                        _DTYPES[dtype], self._ccfg)

    def _workspace(self, device, dtype):
        key = (device.index, dtype)
        ws = self._ws.get(key)
        if ws is None:
            with self._lock:
                ws = self._ws.get(key)
                if ws is None:
                    # zeroed once: status word and piece counters start at zero
                    ws = torch.zeros(self.workspace_bytes(dtype), dtype=torch.uint8, device=device)
                    self._ws[key] = ws
        return ws

    def clock_probe(self, device, dtype) -> tuple:
        """(SM cycles, ns, calls) of the decode kernel accumulated in this workspace
        (see ``MlaDecodeKernel.clock_probe``)."""
        return _clock_probe(self._ws, device, dtype)

    def device_status(self, device, dtype) -> int:
        """Status word the kernel leaves in the workspace (0 = no timeout)."""
        ws = self._ws.get((torch.device(device).index, dtype))
        if ws is None or ws.numel() < 4:
            return 0
        return int(ws[:4].view(torch.int32).item())

    def __call__(self, q, q_pe, kv_cache, k_pe_cache, cache_seqlens, out, lse=None, block_table=None,
                 kv_scale=None):
        """``kv_cache`` may also be an FP8 latent cache (``torch.float8_e4m3fn``, or its bytes
        as ``torch.uint8``) of e4m3 codes whose product with ``kv_scale`` is the latent row
        (mla_decode_ext_fp8kv); ``k_pe_cache`` stays in the model dtype."""
        b, h, smax, ql, kvh = self.batch, self.heads, self.max_seqlen_kv, self.q_len, self.kv_heads
        dtype = q.dtype if isinstance(q, torch.Tensor) else None
        if dtype not in _DTYPES:
            raise ValueError(f"q must be float16 or bfloat16, got {dtype}")
        fp8 = isinstance(kv_cache, torch.Tensor) and kv_cache.dtype in (torch.uint8, _FP8)
        if fp8 and kv_scale is None:
            raise ValueError("an FP8 kv_cache needs kv_scale")
        kv_dtype = kv_cache.dtype if fp8 else dtype
        dev = q.device
        qshape = (b, h) if ql == 1 else (b, ql, h)
        _check_tensor("q", q, (*qshape, DIM), dtype, None)
        _check_tensor("q_pe", q_pe, (*qshape, PE_DIM), dtype, dev)
        _check_tensor("out", out, (*qshape, DIM), dtype, dev)
        sl_ptr = None
        if cache_seqlens is not None:
            _check_tensor("cache_seqlens", cache_seqlens, (b,), torch.int32, dev)
            sl_ptr = cache_seqlens.data_ptr()
        if block_table is None:
            _check_tensor("kv_cache", kv_cache, (b, smax, kvh, DIM), kv_dtype, dev)
            _check_tensor("k_pe_cache", k_pe_cache, (b, smax, kvh, PE_DIM), dtype, dev)
            bt_ptr, page_size, num_pages, max_pages = None, 0, 0, 0
        else:
            if kv_cache.dim() != 4:
                raise ValueError(f"kv_cache must be [num_pages, page_size, {kvh}, 512]")
            num_pages, page_size = int(kv_cache.shape[0]), int(kv_cache.shape[1])
            _check_tensor("kv_cache", kv_cache, (num_pages, page_size, kvh, DIM), kv_dtype, dev)
            _check_tensor("k_pe_cache", k_pe_cache, (num_pages, page_size, kvh, PE_DIM), dtype, dev)
            if block_table.dim() != 2 or block_table.shape[0] != b:
                raise ValueError(f"block_table must be [batch, max_pages], got {tuple(block_table.shape)}")
            max_pages = int(block_table.shape[1])
            _check_tensor("block_table", block_table, (b, max_pages), torch.int32, dev)
            bt_ptr = block_table.data_ptr()
        lse_ptr = None
        if lse is not None:
            _check_tensor("lse", lse, qshape, torch.float32, dev)
            lse_ptr = lse.data_ptr()
        ws = self._workspace(dev, dtype)
        with torch.cuda.device(dev):
            stream = torch.cuda.current_stream(dev).cuda_stream
        if fp8:
            capi.decode_ext_fp8kv(q.data_ptr(), q_pe.data_ptr(), kv_cache.data_ptr(), k_pe_cache.data_ptr(),
                                  float(kv_scale), bt_ptr, sl_ptr, out.data_ptr(), lse_ptr, ws.data_ptr(), ws.numel(),
                                  b, ql, h, kvh, smax, page_size, num_pages, max_pages, _DTYPES[dtype], self._ccfg,
                                  stream)
        else:
            capi.decode_ext(q.data_ptr(), q_pe.data_ptr(), kv_cache.data_ptr(), k_pe_cache.data_ptr(), bt_ptr,
                            sl_ptr, out.data_ptr(), lse_ptr, ws.data_ptr(), ws.numel(), b, ql, h, kvh, smax,
                            page_size, num_pages, max_pages, _DTYPES[dtype], self._ccfg, stream)
