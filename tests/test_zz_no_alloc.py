"""need_gated_scan_noalloc: the gated scan for callers that cannot allocate.

Some callers run the scan where device allocation is not allowed -- an
inference-engine plugin's enqueue step, a serving loop that cannot take
cudaMalloc's device-wide synchronisation, a runtime with a fixed memory
budget.  The no-allocation entry point keeps its look-back scratch in a static
device array inside the library instead of a caller workspace.  These tests
call it through the C ABI and require the same outputs and final state as
need_gated_scan (which uses a workspace) bit for bit -- it is the same kernel
with the same deterministic look-back -- on two calls in a row, with the
first call of the process made on a non-default stream; they read the array's
error word after every call, and check the size limit at exactly the largest
accepted scan and one tile past it.

This file is collected last on purpose; it passes alone in a fresh process and
after the rest of the suite.
"""
import ctypes

import pytest
import torch

from need_b200 import abi
from need_b200 import need_kernels as nk
from need_b200 import workloads

pytestmark = pytest.mark.gpu

SCRATCH_TILES = 2048  # 128-channel tiles of the 16-bit gated scan the static array has records for


def gated_args(w, out, h_final):
    """C-ABI arguments of a [B, T, C] bf16 gated scan with resets and final state."""
    B, T, C = w.x.shape
    a = abi.NeedScanArgs()
    a.form, a.dtype, a.decay_dtype = abi.FORM_GATED, abi.BF16, abi.BF16
    a.nb, a.nh, a.T, a.C = B, 1, T, C
    for k, t in enumerate((w.z, w.g, w.x)):
        a.in_[k] = abi.NeedView(t.data_ptr(), t.stride(0), 0, t.stride(1))
    a.out = out.data_ptr()
    a.out_stride_b, a.out_stride_h, a.out_stride_t = out.stride(0), 0, out.stride(1)
    a.seg_start = w.seg.data_ptr()
    a.seg_stride_b, a.seg_stride_t = w.seg.stride()
    a.h_final = h_final.data_ptr()
    return a


def run_noalloc(lib, w, stream):
    """One need_gated_scan_noalloc call on `stream`; returns (h, h_final, error word)."""
    B, T, C = w.x.shape
    out = torch.full_like(w.x, float("nan"))
    hf = torch.full((B, C), float("nan"), device=w.x.device)
    a = gated_args(w, out, hf)
    a.workspace, a.workspace_bytes = None, 0  # not used by this entry point
    abi.check("need_gated_scan_noalloc", lib.need_gated_scan_noalloc(ctypes.byref(a), stream.cuda_stream))
    err = ctypes.c_uint32(0xffffffff)
    abi.check("need_gated_scan_noalloc_error",
              lib.need_gated_scan_noalloc_error(ctypes.byref(err), stream.cuda_stream))
    return out, hf, int(err.value)


def expect_identical(lib, w, stream, calls=2):
    want, want_f = nk.gated_scan(w.x, w.z, w.g, seg_start=w.seg, return_final_state=True)
    torch.cuda.synchronize()
    for call in range(calls):  # later calls reuse the array the earlier ones left behind
        with torch.cuda.stream(stream):
            got, got_f, err = run_noalloc(lib, w, stream)
        stream.synchronize()
        assert err == 0, f"call {call}: a device-side wait gave up (error bits {err:#x})"
        assert torch.equal(got, want), f"call {call}: outputs differ from need_gated_scan"
        assert torch.equal(got_f, want_f), f"call {call}: final state differs from need_gated_scan"


def test_noalloc_matches_workspace_entry_point_first_call_on_side_stream(cuda):
    """Two calls in a row; the process's first call (which sets the array up)
    runs on a non-default stream, so its zero fill must be ordered on that stream."""
    lib = abi.load()
    side = torch.cuda.Stream(cuda)
    w = workloads.gated_inputs(2, 1000, 512, z_mean=4.0, dtype=torch.bfloat16, device=cuda, seed=21,
                               resets="lognormal", seg_lo=16, seg_hi=400)
    expect_identical(lib, w, side)


def test_noalloc_at_its_largest_scan(cuda):
    """Exactly SCRATCH_TILES tiles (16 chains x 128 chunks), every one after the
    first chunk waiting on look-back records in the static array."""
    lib = abi.load()
    L = lib.need_scan_chunk_len(abi.FORM_GATED, abi.BF16, abi.BF16, 0)
    B, C = 4, 512
    T = SCRATCH_TILES // (B * C // 128) * L
    need = lib.need_scan_workspace_size(abi.FORM_GATED, abi.BF16, abi.BF16, 0, B, 1, T, C)
    assert need == 128 + SCRATCH_TILES * 128 * 32
    w = workloads.gated_inputs(B, T, C, z_mean=4.0, dtype=torch.bfloat16, device=cuda, seed=22,
                               resets="lognormal", seg_lo=16, seg_hi=4096)
    expect_identical(lib, w, torch.cuda.current_stream(cuda))


def test_noalloc_rejects_one_tile_more(cuda):
    lib = abi.load()
    L = lib.need_scan_chunk_len(abi.FORM_GATED, abi.BF16, abi.BF16, 0)
    a = abi.NeedScanArgs()
    a.form, a.dtype = abi.FORM_GATED, abi.BF16
    a.nb, a.nh, a.T, a.C = 1, 1, (SCRATCH_TILES + 1) * L, 128  # one chain of SCRATCH_TILES + 1 chunks
    rc = lib.need_gated_scan_noalloc(ctypes.byref(a), torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == abi.ERR_WORKSPACE
    assert b"static array holds" in lib.need_last_error()
    a.T = SCRATCH_TILES * L  # the same call one tile shorter is accepted by the size check
    assert lib.need_scan_workspace_size(abi.FORM_GATED, abi.BF16, abi.BF16, 0, 1, 1, a.T, 128) == \
        128 + SCRATCH_TILES * 128 * 32
