"""The C ABI without a GPU: the library builds and loads, exports every symbol
include/need_scan.h declares, the ctypes mirror has the header's layout, and
argument errors come back as status codes (these paths make no CUDA call)."""
import ctypes
import os
import re
import subprocess

import pytest

from need_b200 import abi, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "need_scan.h")


@pytest.fixture(scope="module")
def lib():
    build.build()
    return abi.load()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NEED_API\s+[\w\s\*]+?\b(need_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("need_gated_scan", "need_affine_recurrence_scan", "need_ssd_scan", "need_recurrent_retention_scan",
              "need_ragged_verify", "need_commit_states", "need_sp_fixup", "need_scan_workspace_size"):
        assert s in syms
    assert set(syms) == set(abi.SIGNATURES), "ctypes binding and header disagree"


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", build.LIB], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (need_\w+)", out))
    missing = set(declared_symbols()) - exported
    assert not missing, f"not exported: {missing}"
    assert lib.need_abi_version() == abi.ABI_VERSION


def test_struct_layout_matches_header(tmp_path):
    """Compile a C program against the header and compare sizes/offsets with ctypes."""
    fields = {
        "need_scan_args": (abi.NeedScanArgs, [f[0] for f in abi.NeedScanArgs._fields_]),
        "need_verify_args": (abi.NeedVerifyArgs, [f[0] for f in abi.NeedVerifyArgs._fields_]),
        "need_view": (abi.NeedView, [f[0] for f in abi.NeedView._fields_]),
        "need_segment_args": (abi.NeedSegmentArgs, [f[0] for f in abi.NeedSegmentArgs._fields_]),
        "need_conv_args": (abi.NeedConvArgs, [f[0] for f in abi.NeedConvArgs._fields_]),
        "need_ssd_conv": (abi.NeedSsdConv, [f[0] for f in abi.NeedSsdConv._fields_]),
        "need_assoc_args": (abi.NeedAssocArgs, [f[0] for f in abi.NeedAssocArgs._fields_]),
        "need_norm_args": (abi.NeedNormArgs, [f[0] for f in abi.NeedNormArgs._fields_]),
        "need_assoc_step_args": (abi.NeedAssocStepArgs, [f[0] for f in abi.NeedAssocStepArgs._fields_]),
    }
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, (_, names) in fields.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for n in names:
            cn = "in" if n == "in_" else n
            lines.append(f'printf("{cname}.{n} %zu\\n", offsetof({cname}, {cn}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                        check=True).stdout.splitlines())
    for cname, (cls, names) in fields.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
        for n in names:
            assert int(got[f"{cname}.{n}"]) == getattr(cls, n).offset, f"{cname}.{n}"


def test_sizes_and_chunk_lengths(lib):
    L = lib.need_scan_chunk_len(abi.FORM_GATED, abi.BF16, abi.BF16, 0)
    assert L == 128
    ws = lib.need_scan_workspace_size(abi.FORM_GATED, abi.BF16, abi.BF16, 0, 16, 1, 4096, 1024)
    ntiles = 16 * (1024 // 128) * (4096 // L)  # 128-channel tiles
    assert ws == 128 + ntiles * 128 * 32  # header + tagged (A, B) and (prod, h) records per channel
    assert lib.need_scan_workspace_size(abi.FORM_GATED, 7, 7, 0, 1, 1, 1, 8) == 0  # unknown dtype
    # SSD: 64-token tiles of 64 channels (13 channel blocks for C=832)
    assert lib.need_scan_chunk_len(abi.FORM_SSD, abi.BF16, abi.BF16, 0) == 64
    ws = lib.need_scan_workspace_size(abi.FORM_SSD, abi.BF16, abi.BF16, 0, 8, 1, 2048, 832)
    assert ws == 128 + 8 * 13 * (2048 // 64) * 64 * 32
    assert lib.need_scan_chunk_len(abi.FORM_AFFINE, abi.BF16, abi.F16, 0) == -1  # unsupported mix


def test_sequence_parallel_list_size_and_errors(lib):
    """need_sp_list_size: a 4-word count plus one word per gated tile; the
    local scan's argument errors come back before any CUDA call."""
    ntiles = 4 * (4096 // 128) * (8192 // 128)  # B=4, C=4096 (128-channel tiles), T=8192 (128-token chunks)
    assert lib.need_sp_list_size(abi.BF16, 4, 1, 8192, 4096) == 4 + ntiles
    assert lib.need_sp_list_size(7, 4, 1, 8192, 4096) == 0  # unknown dtype
    a = abi.NeedScanArgs()
    assert lib.need_sp_local_scan(None, 1, None) == abi.ERR_INVALID
    assert lib.need_sp_local_scan(ctypes.byref(a), -1, None) == abi.ERR_INVALID
    assert lib.need_sp_local_scan(ctypes.byref(a), 1, None) == abi.ERR_INVALID  # no summary / tile records
    assert b"summary" in lib.need_last_error()


def test_argument_errors_return_status(lib):
    a = abi.NeedScanArgs()
    assert lib.need_gated_scan(None, None) == abi.ERR_INVALID
    assert b"null" in lib.need_last_error()
    a.form = abi.FORM_SSD
    assert lib.need_gated_scan(ctypes.byref(a), None) == abi.ERR_INVALID  # wrong form for the entry point
    a.form = abi.FORM_GATED
    a.dtype = abi.BF16
    a.nb, a.nh, a.T, a.C = 1, 1, 0, 8
    assert lib.need_gated_scan(ctypes.byref(a), None) == abi.ERR_INVALID  # T == 0
    a.T, a.C = 16, 12
    assert lib.need_gated_scan(ctypes.byref(a), None) == abi.ERR_UNSUPPORTED  # C not a multiple of 8
    assert b"multiple of 8" in lib.need_last_error()
    v = abi.NeedVerifyArgs()
    v.form = abi.FORM_AFFINE
    assert lib.need_ragged_verify(ctypes.byref(v), None) == abi.ERR_INVALID
    assert lib.need_commit_states(abi.BF16, 4, 12, None, None, None, None, None, None) == abi.ERR_UNSUPPORTED
    assert lib.need_sp_fixup(None, None, 2, 0, None) == abi.ERR_INVALID
    s = abi.NeedScanArgs()
    s.form, s.dtype, s.nb, s.nh, s.T, s.C = abi.FORM_SSD, abi.BF16, 1, 1, 16, 832
    w = ctypes.c_float(1.0)
    assert lib.need_ssd_scan_rms_norm(None, ctypes.byref(w), abi.F32, 1e-6, None) == abi.ERR_INVALID
    assert lib.need_ssd_scan_rms_norm(ctypes.byref(s), None, abi.F32, 1e-6, None) == abi.ERR_INVALID
    assert lib.need_ssd_scan_rms_norm(ctypes.byref(s), ctypes.byref(w), abi.F16, 1e-6, None) == abi.ERR_UNSUPPORTED
    assert lib.need_ssd_scan_rms_norm(ctypes.byref(s), ctypes.byref(w), abi.F32, -1.0, None) == abi.ERR_INVALID
    cv = abi.NeedSsdConv()
    cv.K, cv.weight = 3, 256
    assert lib.need_ssd_conv_scan(None, ctypes.byref(cv), None, abi.F32, 1e-6, None) == abi.ERR_INVALID
    assert lib.need_ssd_conv_scan(ctypes.byref(s), None, None, abi.F32, 1e-6, None) == abi.ERR_INVALID
    cv.K = 5
    assert lib.need_ssd_conv_scan(ctypes.byref(s), ctypes.byref(cv), None, abi.F32, 1e-6, None) == abi.ERR_UNSUPPORTED
    cv.K, s.dtype = 3, abi.F32
    assert lib.need_ssd_conv_scan(ctypes.byref(s), ctypes.byref(cv), None, abi.F32, 1e-6, None) == abi.ERR_UNSUPPORTED
    s.dtype = abi.BF16
    assert lib.need_ssd_conv_scan(ctypes.byref(s), ctypes.byref(cv), ctypes.byref(w), abi.F16, 1e-6,
                                  None) == abi.ERR_UNSUPPORTED  # norm weight dtype
    s.T = 0
    assert lib.need_ssd_scan_rms_norm(ctypes.byref(s), ctypes.byref(w), abi.F32, 1e-6, None) == abi.ERR_INVALID
    n = abi.NeedNormArgs()
    assert lib.need_rms_norm(None, None) == abi.ERR_INVALID
    n.dtype, n.weight_dtype, n.nb, n.T, n.C = abi.BF16, abi.F32, 1, 4, 832
    assert lib.need_rms_norm(ctypes.byref(n), None) == abi.ERR_INVALID  # null tensors
    n.x = n.out = n.weight = 256
    n.C = 100
    assert lib.need_rms_norm(ctypes.byref(n), None) == abi.ERR_UNSUPPORTED  # C not a multiple of 8
    n.C, n.weight_dtype = 832, abi.F16
    assert lib.need_rms_norm(ctypes.byref(n), None) == abi.ERR_UNSUPPORTED  # weight dtype
    sa = abi.NeedAssocStepArgs()
    assert lib.need_assoc_memory_step(None, None) == abi.ERR_INVALID
    sa.dtype, sa.qk_dtype, sa.nseq, sa.r, sa.d = abi.BF16, abi.F32, 4, 300, 64
    assert lib.need_assoc_memory_step(ctypes.byref(sa), None) == abi.ERR_UNSUPPORTED  # rank above 256
    sa.r = 64
    assert lib.need_assoc_memory_step(ctypes.byref(sa), None) == abi.ERR_INVALID  # null tensors
    m = abi.NeedAssocArgs()
    assert lib.need_assoc_memory(None, None) == abi.ERR_INVALID
    m.dtype, m.qk_dtype, m.nb, m.T, m.r, m.d = abi.BF16, abi.F32, 1, 16, 64, 64
    assert lib.need_assoc_memory(ctypes.byref(m), None) == abi.ERR_INVALID  # null tensors
    m.r = 65
    assert lib.need_assoc_memory(ctypes.byref(m), None) == abi.ERR_UNSUPPORTED  # rank above 64
    m.r, m.dtype = 64, abi.F32
    assert lib.need_assoc_memory(ctypes.byref(m), None) == abi.ERR_UNSUPPORTED  # fp32 values
    assert lib.need_assoc_memory_workspace_size(2, 100, 64, 0) == 128 + 2 * ((2 * 100 * 64 * 2 + 127) // 128 * 128)


def test_assoc_workspace_follows_the_launch_plan(lib):
    """The associative memory's workspace holds the fp32 chunk states of the
    plan the launch will use (B200: 148 SMs; without a GPU the library assumes
    the same).  At d=832 (7 column blocks): 8 sequences of 2048 tokens take two
    segments, the second re-summing the first's tiles, so no chunk states; 4 of
    4096 take 5 segments after 4 chunk states; one of 16384 takes 21 segments
    after 20 chunk states, each [7 blocks][128 columns][64 features] plus z."""

    def feats(nb, t):
        return 2 * ((nb * t * 64 * 2 + 127) // 128 * 128)

    def chunks(n, nb):
        return n * nb * 7 * 128 * 64 * 4 + (n * nb * 64 * 4 + 127) // 128 * 128

    assert lib.need_assoc_memory_workspace_size(8, 2048, 832, 0) == 128 + feats(8, 2048)
    assert lib.need_assoc_memory_workspace_size(4, 4096, 832, 0) == 128 + feats(4, 4096) + chunks(4, 4)
    assert lib.need_assoc_memory_workspace_size(1, 16384, 832, 0) == 128 + feats(1, 16384) + chunks(20, 1)
