"""ctypes binding of ``libmla_decode_b200.so`` (C ABI in include/mla_decode_b200.h).

The library is loaded from this package directory.  There is no fallback:
if it is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

MLA_DTYPE_F16 = 0
MLA_DTYPE_BF16 = 1
MLA_DTYPE_F32 = 2      # output only (mla_combine, mla_decode_partial)

MLA_KERNEL_AUTO = 0
MLA_KERNEL_SIMT = 1
MLA_KERNEL_TC = 2

STATUS_NAMES = {0: "MLA_OK", 1: "MLA_ERR_ARG", 2: "MLA_ERR_WORKSPACE", 3: "MLA_ERR_UNSUPPORTED",
                4: "MLA_ERR_CUDA", 5: "MLA_ERR_DEVICE"}

EXPORTED_SYMBOLS = ("mla_abi_version", "mla_last_error", "mla_split_plan",
                    "mla_workspace_bytes", "mla_decode_fwd", "mla_decode_splitkv",
                    "mla_decode_combine_ws", "mla_combine", "mla_decode_fwd_noalloc",
                    "mla_describe_plan", "mla_decode_partial", "mla_paged_workspace_bytes",
                    "mla_decode_paged", "mla_decode_ext_workspace_bytes", "mla_decode_ext",
                    "mla_decode_fp8kv", "mla_decode_ext_fp8kv", "mla_selftest_wait_timeout",
                    "mla_noalloc_init", "mla_noalloc_status", "mla_combine_strided",
                    "mla_seqsplit_buffer_bytes", "mla_ipc_export", "mla_ipc_import", "mla_ipc_close",
                    "mla_seqsplit_exchange", "mla_seqsplit_decode", "mla_seqsplit_merge")

MLA_SELFTEST_STATUS = 0x1FF   # status word written by mla_selftest_wait_timeout


class MlaCfg(ctypes.Structure):
    """struct MlaCfg (include/mla_decode_b200.h)."""

    _fields_ = [("block_N", ctypes.c_int32), ("block_H", ctypes.c_int32),
                ("num_split", ctypes.c_int32), ("spread", ctypes.c_int32),
                ("num_stages", ctypes.c_int32), ("combine_groups", ctypes.c_int32),
                ("kernel", ctypes.c_int32), ("softmax_scale", ctypes.c_float)]


class MlaError(RuntimeError):
    """A non-zero status returned through the C ABI."""

    def __init__(self, status, message):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True):
    """Load (building first if allowed and needed) and return the CDLL."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if build_if_missing and not _build.up_to_date():
            try:
                _build.build()
            except RuntimeError:
                if not os.path.exists(path):
                    raise
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run `python -m mlc_decode_b200.build`")
        lib = ctypes.CDLL(path)
        vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
        lib.mla_abi_version.argtypes = []
        lib.mla_abi_version.restype = i32
        lib.mla_last_error.argtypes = []
        lib.mla_last_error.restype = ctypes.c_char_p
        lib.mla_split_plan.argtypes = [i32, i32, i32, i32, ctypes.POINTER(i32)]
        lib.mla_split_plan.restype = i32
        lib.mla_workspace_bytes.argtypes = [i32, i32, i32, i32, ctypes.POINTER(MlaCfg)]
        lib.mla_workspace_bytes.restype = sz
        lib.mla_decode_fwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, sz, i32, i32, i32, i32,
                                       ctypes.POINTER(MlaCfg), vp]
        lib.mla_decode_fwd.restype = i32
        lib.mla_decode_splitkv.argtypes = lib.mla_decode_fwd.argtypes
        lib.mla_decode_splitkv.restype = i32
        lib.mla_decode_partial.argtypes = lib.mla_decode_fwd.argtypes
        lib.mla_decode_partial.restype = i32
        lib.mla_paged_workspace_bytes.argtypes = [i32, i32, i32, i32, ctypes.POINTER(MlaCfg)]
        lib.mla_paged_workspace_bytes.restype = sz
        lib.mla_decode_paged.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, i32, i32, i32, i32, i32, i32,
                                         i32, ctypes.POINTER(MlaCfg), vp]
        lib.mla_decode_paged.restype = i32
        lib.mla_decode_fp8kv.argtypes = [vp, vp, vp, vp, ctypes.c_float, vp, vp, vp, sz, i32, i32, i32, i32,
                                         ctypes.POINTER(MlaCfg), vp]
        lib.mla_decode_fp8kv.restype = i32
        lib.mla_decode_ext_fp8kv.argtypes = [vp, vp, vp, vp, ctypes.c_float, vp, vp, vp, vp, vp, sz, i32, i32, i32,
                                             i32, i32, i32, i32, i32, i32, ctypes.POINTER(MlaCfg), vp]
        lib.mla_decode_ext_fp8kv.restype = i32
        lib.mla_selftest_wait_timeout.argtypes = [vp, vp, ctypes.c_uint64, vp]
        lib.mla_selftest_wait_timeout.restype = i32
        lib.mla_decode_ext_workspace_bytes.argtypes = [i32, i32, i32, i32, i32, i32, ctypes.POINTER(MlaCfg)]
        lib.mla_decode_ext_workspace_bytes.restype = sz
        lib.mla_decode_ext.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, i32, i32, i32, i32, i32, i32, i32,
                                       i32, i32, ctypes.POINTER(MlaCfg), vp]
        lib.mla_decode_ext.restype = i32
        lib.mla_decode_combine_ws.argtypes = [vp, vp, vp, sz, i32, i32, i32, i32,
                                              ctypes.POINTER(MlaCfg), vp]
        lib.mla_decode_combine_ws.restype = i32
        lib.mla_decode_fwd_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32,
                                               ctypes.POINTER(MlaCfg), vp]
        lib.mla_decode_fwd_noalloc.restype = i32
        lib.mla_describe_plan.argtypes = [i32, i32, i32, i32, ctypes.POINTER(MlaCfg),
                                           ctypes.POINTER(ctypes.c_int64)]
        lib.mla_describe_plan.restype = i32
        lib.mla_combine.argtypes = [vp, vp, i32, i32, i32, vp, vp, i32, vp]
        lib.mla_combine.restype = i32
        lib.mla_combine_strided.argtypes = [vp, ctypes.c_int64, vp, ctypes.c_int64, i32, i32, i32, vp, vp, i32, vp]
        lib.mla_combine_strided.restype = i32
        lib.mla_noalloc_init.argtypes = []
        lib.mla_noalloc_init.restype = i32
        lib.mla_noalloc_status.argtypes = [vp, vp]
        lib.mla_noalloc_status.restype = i32
        lib.mla_seqsplit_buffer_bytes.argtypes = [i32, i32, i32]
        lib.mla_seqsplit_buffer_bytes.restype = sz
        lib.mla_ipc_export.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint64)]
        lib.mla_ipc_export.restype = i32
        lib.mla_ipc_import.argtypes = [vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]
        lib.mla_ipc_import.restype = i32
        lib.mla_ipc_close.argtypes = [vp, ctypes.c_uint64]
        lib.mla_ipc_close.restype = i32
        lib.mla_seqsplit_exchange.argtypes = [ctypes.POINTER(ctypes.c_void_p), i32, i32, ctypes.c_uint32, i32, i32,
                                              vp]
        lib.mla_seqsplit_exchange.restype = i32
        pvp = ctypes.POINTER(ctypes.c_void_p)
        lib.mla_seqsplit_decode.argtypes = [vp, vp, vp, vp, vp, vp, vp, sz, i32, i32, i32, i32, pvp, i32, i32,
                                            ctypes.c_uint32, ctypes.POINTER(MlaCfg), vp]
        lib.mla_seqsplit_decode.restype = i32
        lib.mla_seqsplit_merge.argtypes = [pvp, i32, i32, ctypes.c_uint32, i32, i32, vp, vp, i32, vp]
        lib.mla_seqsplit_merge.restype = i32
        _lib = lib
        return lib


def last_error() -> str:
    return load().mla_last_error().decode(errors="replace")


def check(status: int):
    if status != 0:
        raise MlaError(status, last_error())


def make_cfg(cfg: dict | None = None, kernel: int | None = None) -> MlaCfg:
    """Map a reference-style config dict (mla_decode.py:588-598) to MlaCfg."""
    cfg = cfg or {}
    c = MlaCfg()
    c.block_N = int(cfg.get("block_N", 0) or 0)
    c.block_H = int(cfg.get("block_H", 0) or 0)
    c.num_split = int(cfg.get("num_split", 0) or 0)
    c.spread = int(bool(cfg.get("spread", False)))
    c.num_stages = int(cfg.get("num_stages", 0) or 0)
    c.combine_groups = int(cfg.get("combine_groups", 1) or 1)
    k = cfg.get("kernel", kernel)
    if isinstance(k, str):
        k = {"auto": MLA_KERNEL_AUTO, "simt": MLA_KERNEL_SIMT, "tc": MLA_KERNEL_TC}[k]
    c.kernel = int(k or 0)
    c.softmax_scale = float(cfg.get("softmax_scale", 0.0) or 0.0)
    return c


def split_plan(seqlen_kv: int, num_split: int, block_n: int, spread: bool = False):
    out = (ctypes.c_int32 * 3)()
    check(load().mla_split_plan(int(seqlen_kv), int(num_split), int(block_n), int(bool(spread)), out))
    return int(out[0]), int(out[1]), int(out[2])


KERNEL_NAMES = {MLA_KERNEL_SIMT: "simt", MLA_KERNEL_TC: "tc"}


def describe_plan(batch, heads, seqlen_kv, dtype, cfg: MlaCfg) -> dict:
    """mla_describe_plan: kernel, splits/pairs, launches per call, zero-prefix bytes."""
    out = (ctypes.c_int64 * 4)()
    check(load().mla_describe_plan(int(batch), int(heads), int(seqlen_kv), int(dtype), ctypes.byref(cfg), out))
    return {"kernel": KERNEL_NAMES.get(int(out[0]), int(out[0])), "splits": int(out[1]),
            "launches": int(out[2]), "zero_prefix_bytes": int(out[3])}


def workspace_bytes(batch, heads, seqlen_kv, dtype, cfg: MlaCfg) -> int:
    n = load().mla_workspace_bytes(int(batch), int(heads), int(seqlen_kv), int(dtype), ctypes.byref(cfg))
    if n == 0:
        msg = last_error()
        if msg:
            raise MlaError(1, msg)
    return int(n)


def decode_fwd(q, q_pe, kv, k_pe, out, lse, ws, ws_bytes, batch, heads, seqlen_kv, dtype,
               cfg: MlaCfg, stream) -> None:
    """Raw pointers in, status checked.  Pointers are ints (device addresses)."""
    check(load().mla_decode_fwd(q, q_pe, kv, k_pe, out, lse, ws, ws_bytes, int(batch), int(heads),
                                int(seqlen_kv), int(dtype), ctypes.byref(cfg), stream))


def decode_fwd_noalloc(q, q_pe, kv, k_pe, out, lse, batch, heads, seqlen_kv, dtype, cfg: MlaCfg,
                       stream) -> None:
    """mla_decode_fwd_noalloc: scratch from the library's static device array (no allocation)."""
    check(load().mla_decode_fwd_noalloc(q, q_pe, kv, k_pe, out, lse, int(batch), int(heads),
                                        int(seqlen_kv), int(dtype), ctypes.byref(cfg), stream))


def decode_partial(q, q_pe, kv, k_pe, o, lse, ws, ws_bytes, batch, heads, seqlen_kv, dtype,
                   cfg: MlaCfg, stream) -> None:
    """mla_decode_partial: float32 normalised O and natural-log LSE of this KV part."""
    check(load().mla_decode_partial(q, q_pe, kv, k_pe, o, lse, ws, ws_bytes, int(batch), int(heads),
                                    int(seqlen_kv), int(dtype), ctypes.byref(cfg), stream))


def paged_workspace_bytes(batch, heads, max_seqlen_kv, dtype, cfg: MlaCfg) -> int:
    lib = load()
    n = lib.mla_paged_workspace_bytes(int(batch), int(heads), int(max_seqlen_kv), int(dtype), ctypes.byref(cfg))
    if n == 0:
        msg = last_error()
        if msg:
            raise MlaError(1, msg)
    return int(n)


def decode_paged(q, q_pe, kv_cache, k_pe_cache, block_table, cache_seqlens, out, lse, ws, ws_bytes, batch,
                 heads, max_seqlen_kv, page_size, num_pages, max_pages, dtype, cfg: MlaCfg, stream) -> None:
    """mla_decode_paged: per-sequence KV lengths, optional page table (pointers are device addresses)."""
    check(load().mla_decode_paged(q, q_pe, kv_cache, k_pe_cache, block_table, cache_seqlens, out, lse, ws,
                                  ws_bytes, int(batch), int(heads), int(max_seqlen_kv), int(page_size),
                                  int(num_pages), int(max_pages), int(dtype), ctypes.byref(cfg), stream))


def decode_fp8kv(q, q_pe, kv_fp8, k_pe, kv_scale, out, lse, ws, ws_bytes, batch, heads, seqlen_kv, dtype,
                 cfg: MlaCfg, stream) -> None:
    """mla_decode_fp8kv: e4m3 latent KV rows times kv_scale (pointers are device addresses)."""
    check(load().mla_decode_fp8kv(q, q_pe, kv_fp8, k_pe, float(kv_scale), out, lse, ws, ws_bytes, int(batch),
                                  int(heads), int(seqlen_kv), int(dtype), ctypes.byref(cfg), stream))


def selftest_wait_timeout(status, result, limit_ns, stream) -> None:
    """mla_selftest_wait_timeout: the decode kernel's bounded-wait path run on barriers
    nothing arrives on (status: device uint32 word, zero before; result: device 4 x uint64)."""
    check(load().mla_selftest_wait_timeout(status, result, int(limit_ns), stream))


def ext_workspace_bytes(batch, q_len, heads, kv_heads, max_seqlen_kv, dtype, cfg: MlaCfg) -> int:
    lib = load()
    n = lib.mla_decode_ext_workspace_bytes(int(batch), int(q_len), int(heads), int(kv_heads), int(max_seqlen_kv),
                                           int(dtype), ctypes.byref(cfg))
    if n == 0:
        msg = last_error()
        if msg:
            raise MlaError(1, msg)
    return int(n)


def decode_ext(q, q_pe, kv_cache, k_pe_cache, block_table, cache_seqlens, out, lse, ws, ws_bytes, batch, q_len,
               heads, kv_heads, max_seqlen_kv, page_size, num_pages, max_pages, dtype, cfg: MlaCfg, stream) -> None:
    """mla_decode_ext: q_len query positions per sequence (causal within the step), kv_heads KV heads,
    per-sequence KV lengths (cache_seqlens may be None) and an optional page table."""
    check(load().mla_decode_ext(q, q_pe, kv_cache, k_pe_cache, block_table, cache_seqlens, out, lse, ws, ws_bytes,
                                int(batch), int(q_len), int(heads), int(kv_heads), int(max_seqlen_kv),
                                int(page_size), int(num_pages), int(max_pages), int(dtype), ctypes.byref(cfg),
                                stream))


def decode_ext_fp8kv(q, q_pe, kv_fp8, k_pe_cache, kv_scale, block_table, cache_seqlens, out, lse, ws, ws_bytes,
                     batch, q_len, heads, kv_heads, max_seqlen_kv, page_size, num_pages, max_pages, dtype,
                     cfg: MlaCfg, stream) -> None:
    """mla_decode_ext_fp8kv: mla_decode_ext over an e4m3 latent cache times kv_scale."""
    check(load().mla_decode_ext_fp8kv(q, q_pe, kv_fp8, k_pe_cache, float(kv_scale), block_table, cache_seqlens, out,
                                      lse, ws, ws_bytes, int(batch), int(q_len), int(heads), int(kv_heads),
                                      int(max_seqlen_kv), int(page_size), int(num_pages), int(max_pages), int(dtype),
                                      ctypes.byref(cfg), stream))


def decode_splitkv(q, q_pe, kv, k_pe, out, lse, ws, ws_bytes, batch, heads, seqlen_kv, dtype,
                   cfg: MlaCfg, stream) -> None:
    check(load().mla_decode_splitkv(q, q_pe, kv, k_pe, out, lse, ws, ws_bytes, int(batch), int(heads),
                                    int(seqlen_kv), int(dtype), ctypes.byref(cfg), stream))


def decode_combine_ws(out, lse, ws, ws_bytes, batch, heads, seqlen_kv, dtype, cfg: MlaCfg,
                      stream) -> None:
    check(load().mla_decode_combine_ws(out, lse, ws, ws_bytes, int(batch), int(heads), int(seqlen_kv),
                                       int(dtype), ctypes.byref(cfg), stream))


def combine(part_lse, part_o, num_split, batch, heads, out, lse, dtype, stream) -> None:
    check(load().mla_combine(part_lse, part_o, int(num_split), int(batch), int(heads), out, lse,
                             int(dtype), stream))


def combine_strided(part_lse, lse_stride, part_o, o_stride, num_split, batch, heads, out, lse, dtype,
                    stream) -> None:
    """mla_combine_strided: split k's rows at part_lse + k*lse_stride, part_o + k*o_stride (floats)."""
    check(load().mla_combine_strided(part_lse, int(lse_stride), part_o, int(o_stride), int(num_split),
                                     int(batch), int(heads), out, lse, int(dtype), stream))


def noalloc_init() -> None:
    """mla_noalloc_init: look up the static scratch array on the current device."""
    check(load().mla_noalloc_init())


def noalloc_status(status_out, stream) -> None:
    """mla_noalloc_status: enqueue a copy of the static array's status word to ``status_out``."""
    check(load().mla_noalloc_status(status_out, stream))


def seqsplit_buffer_bytes(world, batch, heads) -> int:
    n = load().mla_seqsplit_buffer_bytes(int(world), int(batch), int(heads))
    if n == 0:
        raise MlaError(1, last_error())
    return int(n)


def ipc_export(ptr) -> tuple[bytes, int]:
    """CUDA IPC handle (64 bytes) of the allocation holding device pointer ``ptr``, and
    ``ptr``'s offset in it."""
    h = (ctypes.c_char * 64)()
    off = ctypes.c_uint64()
    check(load().mla_ipc_export(ptr, h, ctypes.byref(off)))
    return bytes(h), int(off.value)


def ipc_import(handle: bytes, offset: int) -> int:
    """Device pointer, in this process, of a peer's memory exported by ``ipc_export``."""
    h = (ctypes.c_char * 64).from_buffer_copy(handle)
    p = ctypes.c_void_p()
    check(load().mla_ipc_import(h, int(offset), ctypes.byref(p)))
    return int(p.value)


def ipc_close(ptr, offset) -> None:
    check(load().mla_ipc_close(ptr, int(offset)))


def seqsplit_exchange(bufs, world, rank, epoch, batch, heads, stream) -> None:
    arr = (ctypes.c_void_p * len(bufs))(*bufs)
    check(load().mla_seqsplit_exchange(arr, int(world), int(rank), int(epoch), int(batch), int(heads), stream))


def seqsplit_exchange_raw(arr, world, rank, epoch, batch, heads, stream) -> None:
    """seqsplit_exchange with the buffers already as a ctypes c_void_p array."""
    check(load().mla_seqsplit_exchange(arr, int(world), int(rank), int(epoch), int(batch), int(heads), stream))


def seqsplit_decode(q, q_pe, kv_part, k_pe_part, out, lse, ws, ws_bytes, batch, heads, seqlen_part, dtype, bufs,
                    world, rank, epoch, cfg: MlaCfg, stream) -> None:
    """mla_seqsplit_decode: this rank's decode, then the row-wise exchange and merge.

    ``bufs``: every rank's gather buffer pointer, a sequence or a ctypes c_void_p array.
    """
    arr = bufs if isinstance(bufs, ctypes.Array) else (ctypes.c_void_p * len(bufs))(*bufs)
    check(load().mla_seqsplit_decode(q, q_pe, kv_part, k_pe_part, out, lse, ws, ws_bytes, int(batch), int(heads),
                                     int(seqlen_part), int(dtype), arr, int(world), int(rank), int(epoch),
                                     ctypes.byref(cfg), stream))


def seqsplit_merge(bufs, world, rank, epoch, batch, heads, out, lse, dtype, stream) -> None:
    """mla_seqsplit_merge: the row-wise exchange and merge of blocks already written."""
    arr = bufs if isinstance(bufs, ctypes.Array) else (ctypes.c_void_p * len(bufs))(*bufs)
    check(load().mla_seqsplit_merge(arr, int(world), int(rank), int(epoch), int(batch), int(heads), out, lse,
                                    int(dtype), stream))
