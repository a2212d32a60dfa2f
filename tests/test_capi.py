"""The C-ABI library loads, exports every declared symbol, and its host logic
(split planner, workspace sizing, argument checks) is right.  No GPU needed:
nothing here launches a kernel."""
import ctypes
import glob
import json
import os
import re

import pytest

from mlc_decode_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(mla_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    return capi.load()


def test_library_exports_every_declared_symbol(lib):
    declared = _declared_functions()
    assert set(capi.EXPORTED_SYMBOLS) <= set(declared)
    for name in declared:
        assert hasattr(lib, name), name


def test_abi_version(lib):
    assert lib.mla_abi_version() == 1


def test_split_plan_c_matches_reference_golden():
    with open(os.path.join(ROOT, "tests", "golden", "split_plan.json")) as f:
        plans = json.load(f)
    for s, ns, bn, spread, expect in plans:
        assert list(capi.split_plan(s, ns, bn, bool(spread))) == expect, (s, ns, bn, spread)


def test_workspace_bytes_simt_formula():
    cfg = capi.make_cfg({"kernel": "simt", "block_N": 32, "num_split": 64})
    n = capi.workspace_bytes(2, 16, 8192, capi.MLA_DTYPE_F16, cfg)
    ns = capi.split_plan(8192, 64, 32, False)[0]
    rows = ns * 2 * 16
    assert n == -(-rows * 4 // 256) * 256 + rows * 512 * 4
    one = capi.make_cfg({"kernel": "simt", "block_N": 32, "num_split": 1})
    assert capi.workspace_bytes(2, 16, 8192, capi.MLA_DTYPE_F16, one) == 0


def test_bad_arguments_return_codes_without_touching_the_gpu(lib):
    cfg = capi.make_cfg({})
    fwd = lib.mla_decode_fwd
    # null pointers
    rc = fwd(None, None, None, None, None, None, None, 0, 1, 16, 64, 1, ctypes.byref(cfg), None)
    assert rc == 1 and "null" in capi.last_error()
    # bad shape
    rc = fwd(16, 16, 16, 16, 16, None, None, 0, 0, 16, 64, 1, ctypes.byref(cfg), None)
    assert rc == 1 and ">= 1" in capi.last_error()
    # bad dtype
    rc = fwd(16, 16, 16, 16, 16, None, None, 0, 1, 16, 64, 7, ctypes.byref(cfg), None)
    assert rc == 1 and "dtype" in capi.last_error()
    # misaligned pointer
    rc = fwd(18, 16, 16, 16, 16, None, None, 0, 1, 16, 64, 1, ctypes.byref(cfg), None)
    assert rc == 1 and "aligned" in capi.last_error()
    # workspace too small
    big = capi.make_cfg({"kernel": "simt", "num_split": 8})
    rc = fwd(256, 256, 256, 256, 256, None, 256, 16, 1, 16, 4096, 1, ctypes.byref(big), None)
    assert rc == 2 and "workspace" in capi.last_error()
    # unknown kernel kind
    odd = capi.make_cfg({"kernel": 9})
    rc = fwd(256, 256, 256, 256, 256, None, 256, 1 << 30, 1, 16, 64, 1, ctypes.byref(odd), None)
    assert rc == 1
    # bad softmax scale
    neg = capi.make_cfg({"kernel": "simt", "num_split": 1, "softmax_scale": -1.0})
    rc = fwd(256, 256, 256, 256, 256, None, None, 0, 1, 16, 64, 1, ctypes.byref(neg), None)
    assert rc == 1 and "softmax_scale" in capi.last_error()


def test_combine_argument_checks(lib):
    rc = lib.mla_combine(None, None, 1, 1, 1, None, None, 0, None)
    assert rc == 1
    rc = lib.mla_combine(256, 256, 0, 1, 1, 256, None, 0, None)
    assert rc == 1
    rc = lib.mla_combine(256, 260, 2, 1, 1, 256, None, 0, None)
    assert rc == 1 and "aligned" in capi.last_error()


def test_error_text_is_thread_local(lib):
    import threading

    cfg = capi.make_cfg({})
    lib.mla_decode_fwd(None, None, None, None, None, None, None, 0, 1, 16, 64, 1, ctypes.byref(cfg), None)
    seen = {}

    def other():
        seen["msg"] = capi.last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""
    assert "null" in capi.last_error()


def test_drop_in_module_surface():
    import mla_decode

    for name in ("_get_kernel", "run_kernel", "build_kernel_from_config", "mla_autotune_configs",
                 "_split_plan", "flashattn_shared_q", "flashattn_frag_q", "flashattn_autotuned",
                 "_legacy_kernel", "_TUNE_CACHE", "_AUTOTUNE_ENABLED"):
        assert hasattr(mla_decode, name), name
    assert mla_decode._split_plan(8192, 64, 32) == (64, 4, 0)
    assert mla_decode._split_plan(16384, 104, 32, True) == (104, 4, 96)
    cfgs = mla_decode.mla_autotune_configs(64, 128, 1, 8192, 512, 64)
    assert cfgs and all({"block_N", "num_split", "spread"} <= set(c) for c in cfgs)


def test_kernel_object_rejects_non_absorbed_shapes():
    from mlc_decode_b200 import MlaDecodeKernel

    with pytest.raises(ValueError):
        MlaDecodeKernel(1, 16, 3, 64, 512, 64)    # heads not a multiple of kv_head_num
    with pytest.raises(ValueError):
        MlaDecodeKernel(1, 16, 2, 64, 512, 64, cfg={"kernel": "simt"})
    with pytest.raises(ValueError):
        MlaDecodeKernel(1, 16, 1, 64, 256, 64)
    k = MlaDecodeKernel(1, 16, 2, 64, 512, 64)   # grouped KV heads: the mla_decode_ext path
    with pytest.raises(NotImplementedError):
        k.plan()


def test_seqsplit_buffer_layout_sizes(lib):
    """mla_seqsplit_buffer_bytes: float32 (O, LSE) blocks [2][world][chunk], a 256-byte
    header, then (value, call number) words for rows and LSEs; world 1..8."""
    for world in range(1, 9):
        for b, h in ((1, 128), (3, 64), (2, 16), (5, 200)):
            bh = b * h
            rows_pad = -(-bh // 64) * 64
            chunk = bh * 512 + rows_pad
            header = -(-2 * world * chunk * 4 // 256) * 256
            ll_lse = header + 256 + 2 * world * rows_pad * 512 * 8
            assert capi.seqsplit_buffer_bytes(world, b, h) == ll_lse + 2 * world * rows_pad * 8
    for bad in ((0, 1, 128), (9, 1, 128), (2, 0, 128), (2, 1, 0)):
        assert lib.mla_seqsplit_buffer_bytes(*bad) == 0


def test_seqsplit_entry_points_reject_bad_arguments_without_touching_the_gpu(lib):
    cfg = capi.make_cfg({})
    arr = (ctypes.c_void_p * 2)(256, 512)
    dec = lib.mla_seqsplit_decode
    # world out of range, rank outside the world, call number 0, no buffers
    for world, rank, epoch, bufs in ((0, 0, 1, arr), (9, 0, 1, arr), (2, 2, 1, arr), (2, 0, 0, arr), (2, 0, 1, None)):
        rc = dec(256, 256, 256, 256, 256, None, 256, 1 << 20, 1, 128, 1024, 1, bufs, world, rank, epoch,
                 ctypes.byref(cfg), None)
        assert rc == 1 and "bad argument" in capi.last_error(), (world, rank, epoch)
    # a buffer that is not 256-byte aligned
    odd = (ctypes.c_void_p * 2)(256, 528)
    rc = dec(256, 256, 256, 256, 256, None, 256, 1 << 20, 1, 128, 1024, 1, odd, 2, 0, 1, ctypes.byref(cfg), None)
    assert rc == 1 and "256-byte" in capi.last_error()
    # a null or misaligned output
    rc = dec(256, 256, 256, 256, None, None, 256, 1 << 20, 1, 128, 1024, 1, arr, 2, 0, 1, ctypes.byref(cfg), None)
    assert rc == 1 and "out" in capi.last_error()
    mrg = lib.mla_seqsplit_merge
    assert mrg(arr, 2, 0, 1, 1, 128, 264, None, 1, None) == 1 and "aligned" in capi.last_error()
    assert mrg(arr, 2, 0, 1, 1, 128, 256, None, 7, None) == 1 and "dtype" in capi.last_error()
    assert mrg(arr, 2, 5, 1, 1, 128, 256, None, 1, None) == 1 and "bad argument" in capi.last_error()
