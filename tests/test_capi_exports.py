"""The C-ABI library loads on a machine without a GPU and exports every entry
point declared in include/polylora_b200.h.  Only argument checks that return
before any CUDA call are exercised here."""

import ctypes
import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parents[1] / "include" / "polylora_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(plora_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for required in ("plora_sgmv_a_fwd", "plora_sgmv_b_fwd", "plora_sgmv_shrink", "plora_sgmv_expand",
                     "plora_build_segments", "plora_flat_schedule", "plora_slot_fill",
                     "plora_workspace_size", "plora_device_status"):
        assert required in names


def test_library_exports_every_declared_symbol(native):
    lib = native.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # the ctypes binding covers the whole header
    assert set(declared_functions()) <= set(native._SIGNATURES)


def test_weight_split_threshold_round_trips(native):
    """The work-split threshold is host state: set, read back, restored."""
    prev = native.weight_split_tokens_per_sm(7)
    try:
        assert prev >= 0
        assert native.weight_split_tokens_per_sm() == 7
        assert native.weight_split_tokens_per_sm(0) == 7
        assert native.weight_split_tokens_per_sm(-5) == 0  # negative: query only
    finally:
        native.weight_split_tokens_per_sm(prev)
    assert native.weight_split_tokens_per_sm() == prev


def test_version_and_status_strings(native):
    assert "sm_100a" in native.version()
    lib = native.load()
    assert lib.plora_status_string(native.OK) == b"ok"
    assert lib.plora_status_string(native.ERR_WORKSPACE) == b"workspace too small"


def test_struct_layouts_match_header(native):
    assert ctypes.sizeof(native.SlotModule) == 48
    assert ctypes.sizeof(native.SlotRecord) == 24


@pytest.mark.parametrize("dtype", [3, -1])
def test_bad_dtype_rejected_before_cuda(native, dtype):
    lib = native.load()
    st = lib.plora_sgmv_shrink(None, None, None, None, None, None, 16, 64, 16, 5, 1, dtype, None)
    assert st == native.ERR_INVALID_ARGUMENT
    assert "dtype" in native.last_error()


def test_workspace_size_and_null_checks(native):
    lib = native.load()
    assert native.workspace_size(16384, 1, 65) >= (16384 + 66) * 4
    assert native.workspace_size(-1, 1, 65) == 0
    # too many slots is refused up front
    st = lib.plora_sgmv_expand(None, None, None, None, None, None, None, 8, 16, 64, 5000, 2, None)
    assert st == native.ERR_UNSUPPORTED
    # missing workspace
    st = lib.plora_sgmv_a_fwd(None, None, None, None, None, None, 4, 2, 64, 16, 5, 1, 2, None, 0, None)
    assert st == native.ERR_WORKSPACE
    # the combined shrink + expand checks its arguments before any CUDA call
    st = lib.plora_sgmv_shrink_expand(None, None, None, None, None, None, None, None, None,
                                      8, 64, 16, 64, 5, 2, None)
    assert st == native.ERR_INVALID_ARGUMENT and "null" in native.last_error()
    st = lib.plora_sgmv_shrink_expand(None, None, None, None, None, None, None, None, None,
                                      8, 0, 16, 64, 5, 2, None)
    assert st == native.ERR_INVALID_ARGUMENT


def test_product_path_has_no_cpu_fallback():
    import torch

    from polylora_b200.sgmv import sgmv_lora_a_fwd

    x = torch.zeros(2, 3, 8)
    w = torch.zeros(3, 8, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        sgmv_lora_a_fwd(x, w, torch.ones(2, dtype=torch.int32), torch.zeros(2, dtype=torch.int64),
                        torch.zeros(3, dtype=torch.int32))
    from polylora_b200.host_io import HostLoraPipeline

    with pytest.raises(RuntimeError, match="no CPU fallback"):
        HostLoraPipeline("cpu")


def test_segment_and_slot_fill_limits_rejected_before_cuda(native):
    """Size limits and slot-fill arguments are checked on the host, before any
    CUDA call (the non-null pointers below are never dereferenced)."""
    lib = native.load()
    dummy = 0x1000
    # more slots than the segment kernels take
    st = lib.plora_build_segments(dummy, dummy, dummy, 4, 1, 5000, dummy, dummy, dummy, 1 << 20, None)
    assert st == native.ERR_UNSUPPORTED and "num_slots" in native.last_error()
    # token ids must fit in int32
    st = lib.plora_build_segments(dummy, dummy, dummy, 1 << 20, 1 << 12, 65, dummy, dummy, dummy, 1 << 20, None)
    assert st == native.ERR_UNSUPPORTED and "int32" in native.last_error()
    # slot fill: slot outside the cache, image smaller than its records, staging too small
    fill = lambda slot, image_bytes, staging_bytes: lib.plora_slot_fill(  # noqa: E731
        dummy, 2, slot, 4, 16, native.DTYPE_BF16, dummy, image_bytes, dummy, staging_bytes, None)
    assert fill(4, 4096, 4096) == native.ERR_INVALID_ARGUMENT
    assert fill(1, 47, 4096) == native.ERR_INVALID_ARGUMENT and "records" in native.last_error()
    assert fill(1, 4096, 4095) == native.ERR_WORKSPACE


def test_padding_check_arguments_rejected_before_cuda(native):
    """plora_check_right_padded checks element sizes, shapes and alignment on
    the host; an empty mask returns at once."""
    lib = native.load()
    dummy = 0x1000
    assert lib.plora_check_right_padded(dummy, 3, 0, dummy, 2, 2, None) == native.ERR_INVALID_ARGUMENT
    assert lib.plora_check_right_padded(dummy, 1, 1, dummy, 2, 2, None) == native.ERR_INVALID_ARGUMENT
    assert lib.plora_check_right_padded(dummy, 8, 0, dummy, -1, 2, None) == native.ERR_INVALID_ARGUMENT
    assert lib.plora_check_right_padded(dummy + 2, 4, 0, dummy, 2, 2, None) == native.ERR_INVALID_ARGUMENT
    assert "aligned" in native.last_error()
    assert lib.plora_check_right_padded(None, 8, 0, None, 2, 2, None) == native.ERR_INVALID_ARGUMENT
    assert lib.plora_check_right_padded(None, 8, 0, None, 0, 7, None) == native.OK
    assert lib.plora_check_right_padded(None, 2, 1, None, 5, 0, None) == native.OK


def test_header_is_plain_c_and_links(tmp_path, native):
    """A C11 program that includes the header (pedantic, warnings as errors),
    takes the address of every declared entry point and links against the
    library: the boundary is a C ABI, usable without C++ or CUDA headers."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = Path(native.load()._name)
    names = declared_functions()
    src = tmp_path / "caller.c"
    src.write_text(
        '#include "polylora_b200.h"\n#include <stdio.h>\n'
        "typedef void (*fn)(void);\n"
        "_Static_assert(sizeof(plora_slot_module) == 48, \"plora_slot_module layout\");\n"
        "_Static_assert(sizeof(plora_slot_record) == 24, \"plora_slot_record layout\");\n"
        "static const fn entry_points[] = {\n" + ",\n".join(f"  (fn){n}" for n in names) + "\n};\n"
        'int main(void) { printf("%d\\n", (int)(sizeof entry_points / sizeof entry_points[0])); return 0; }\n')
    out = tmp_path / "caller"
    res = subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{HEADER.parent}", str(src),
                          f"-L{lib.parent}", f"-l:{lib.name}", f"-Wl,-rpath,{lib.parent}", "-o", str(out)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(out)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == str(len(names)), run.stderr


@pytest.mark.parametrize("rows,seq", [(1 << 18, 1 << 46), (1 << 40, 1 << 30), (3, -1), (-2, 5), (1 << 31, 1)])
def test_token_count_overflow_rejected_before_cuda(native, rows, seq):
    """num_rows x max_seq that overflows int64 (e.g. 2^18 x 2^46 wraps to 0), is
    negative, or exceeds int32 token ids is refused by every entry point that
    sizes scratch from it, before any CUDA call: no scratch carve can then run
    past its buffer."""
    lib = native.load()
    dummy = 0x1000
    assert native.workspace_size(rows, seq, 65) == 0
    st = lib.plora_sgmv_a_fwd_noalloc(dummy, dummy, dummy, dummy, dummy, dummy, rows, seq, 64, 16, 65, 1,
                                      native.DTYPE_BF16, None)
    assert st in (native.ERR_UNSUPPORTED, native.ERR_INVALID_ARGUMENT), native.last_error()
    st = lib.plora_sgmv_a_fwd(dummy, dummy, dummy, dummy, dummy, dummy, rows, seq, 64, 16, 65, 1,
                              native.DTYPE_BF16, dummy, 1 << 30, None)
    assert st in (native.ERR_UNSUPPORTED, native.ERR_INVALID_ARGUMENT), native.last_error()
    st = lib.plora_sgmv_b_fwd(dummy, dummy, dummy, dummy, dummy, dummy, dummy, rows, seq, 16, 64, 65,
                              native.DTYPE_BF16, dummy, 1 << 30, None)
    assert st in (native.ERR_UNSUPPORTED, native.ERR_INVALID_ARGUMENT), native.last_error()
    st = lib.plora_build_segments(dummy, dummy, dummy, rows, seq, 65, dummy, dummy, dummy, 1 << 30, None)
    assert st in (native.ERR_UNSUPPORTED, native.ERR_INVALID_ARGUMENT), native.last_error()


def test_stream_kernel_switch_round_trips(native):
    prev = native.stream_kernels()
    try:
        assert prev == 2  # the default: stream kernels, the combined call fused
        assert native.stream_kernels(0) == prev
        assert native.stream_kernels() == 0
        assert native.stream_kernels(1) == 0
        assert native.stream_kernels(5) == 1  # values above 2 mean 2
        assert native.stream_kernels() == 2
    finally:
        native.stream_kernels(prev)


def test_token_rows_arguments_rejected_before_cuda(native):
    """plora_gather_token_rows / plora_scatter_token_rows check row sizes,
    counts, slots, nulls and alignment on the host; no tokens returns at once."""
    lib = native.load()
    dummy = 0x1000
    for fn in (lib.plora_gather_token_rows, lib.plora_scatter_token_rows):
        assert fn(dummy, dummy, 24, 4, dummy, dummy, 1, None) == native.ERR_INVALID_ARGUMENT  # not a multiple of 16
        assert "multiple of 16" in native.last_error()
        assert fn(dummy, dummy, 0, 4, dummy, dummy, 1, None) == native.ERR_INVALID_ARGUMENT
        assert fn(dummy, dummy, 32, -1, dummy, dummy, 1, None) == native.ERR_INVALID_ARGUMENT
        assert fn(dummy, dummy, 32, 4, dummy, dummy, 0, None) == native.ERR_UNSUPPORTED
        assert fn(dummy, dummy, 32, 1 << 32, dummy, dummy, 1, None) == native.ERR_UNSUPPORTED
        assert fn(dummy, dummy, 1 << 40, 1 << 30, dummy, dummy, 1, None) == native.ERR_INVALID_ARGUMENT  # overflow
        assert fn(None, dummy, 32, 4, dummy, dummy, 1, None) == native.ERR_INVALID_ARGUMENT
        assert fn(dummy + 8, dummy, 32, 4, dummy, dummy, 1, None) == native.ERR_INVALID_ARGUMENT
        assert "aligned" in native.last_error()
        assert fn(None, None, 32, 0, None, None, 1, None) == native.OK
