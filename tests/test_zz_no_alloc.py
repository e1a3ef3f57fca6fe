"""need_gated_scan_noalloc: the gated scan for callers that cannot allocate.

Some callers run the scan where device allocation is not allowed -- an
inference-engine plugin's enqueue step, a serving loop that cannot take
cudaMalloc's device-wide synchronisation, a runtime with a fixed memory
budget.  The no-allocation entry point keeps its look-back scratch in a static
device array inside the library instead of a caller workspace.  These tests
call it through the C ABI and check it against need_gated_scan (which uses a
workspace), on two calls in a row, with the tolerance of the other bf16 tests.

This file is collected last on purpose; it passes alone in a fresh process and
after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

from need_b200 import abi
from need_b200 import need_kernels as nk
from need_b200 import workloads

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


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


def test_noalloc_matches_workspace_entry_point(cuda):
    lib = abi.load()
    w = workloads.gated_inputs(2, 1000, 512, z_mean=4.0, dtype=torch.bfloat16, device=cuda, seed=21,
                               resets="lognormal", seg_lo=16, seg_hi=400)
    want, want_f = nk.gated_scan(w.x, w.z, w.g, seg_start=w.seg, return_final_state=True)
    want_h, want_fh = want.float().cpu().numpy(), want_f.cpu().numpy()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call in range(2):  # the second call reuses the array the first one left behind
        out = torch.full_like(w.x, float("nan"))
        hf = torch.full((2, 512), float("nan"), device=cuda)
        a = gated_args(w, out, hf)
        a.workspace, a.workspace_bytes = None, 0  # not used by this entry point
        abi.check("need_gated_scan_noalloc", lib.need_gated_scan_noalloc(ctypes.byref(a), stream))
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: unwritten outputs"
        err = np.abs(got - want_h).max() / np.abs(want_h).max()
        assert err <= BF16_TOL, f"call {call}: rel err {err}"
        assert np.mean(got == want_h) >= 0.99, f"call {call}: outputs differ from need_gated_scan"
        ferr = np.abs(hf.cpu().numpy() - want_fh).max() / np.abs(want_fh).max()
        assert ferr <= 1e-5, f"call {call}: final state rel err {ferr}"


def test_noalloc_rejects_scans_larger_than_its_scratch(cuda):
    lib = abi.load()
    a = abi.NeedScanArgs()
    a.form, a.dtype = abi.FORM_GATED, abi.BF16
    a.nb, a.nh, a.T, a.C = 16, 1, 65536, 1024  # 16384 tiles > 1024
    rc = lib.need_gated_scan_noalloc(ctypes.byref(a), torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == abi.ERR_WORKSPACE
    assert b"static array holds" in lib.need_last_error()
