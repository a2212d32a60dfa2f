"""bench.py's command line: workload defaults per mode (no GPU needed)."""
import sys

import pytest

import bench


def parse(argv):
    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench.parse_args()
    finally:
        sys.argv = old


def test_default_workload_is_configs1():
    a = parse([])
    assert (a.batch, a.heads, a.kv_ctx, a.dtype, a.gpus) == (64, 128, 8192, "bf16", 1)
    assert not a.seq_split


def test_seq_split_defaults_to_configs4b():
    a = parse(["--seq-split", "--gpus", "8"])
    assert (a.batch, a.heads, a.kv_ctx) == (1, 128, 131072)
    assert "split across 8 GPU(s)" in bench.workload_name(a)


def test_seq_split_keeps_explicit_shape():
    a = parse(["--seq-split", "--batch", "2", "--kv-ctx", "65536"])
    assert (a.batch, a.kv_ctx) == (2, 65536)


@pytest.mark.parametrize("extra", [["--fp8"], ["--paged", "64"]])
def test_seq_split_rejects_other_modes(extra):
    with pytest.raises(SystemExit):
        parse(["--seq-split", *extra])


def test_roofline_numbers():
    by, fl = bench.algorithmic(64, 128, 8192)
    assert by == 603_979_776 and fl == 2.0 * 64 * 128 * 8192 * 1088
    by8, _ = bench.algorithmic(64, 128, 8192, fp8=True)
    assert by8 == 64 * 8192 * (512 + 128)
