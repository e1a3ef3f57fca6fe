"""A bounded device-side wait that runs out: the launch completes, the error is
reported through the workspace's error word, and the context stays usable.

Every look-back wait in the scan kernel is bounded: after the poll limit it
sets ERR_LOOKBACK in the workspace's error word, takes a zero carry and lets
the launch finish.  The test hook need_test_set_lookback_polls lowers that
limit to 4 polls -- far less than the microseconds a tile's predecessors need
just to load their rows -- so the look-back waits of the launch run out (the
records they wait for are published only later, as a flag that is not set in
time would be).  Nothing is read or written out of bounds and every wait ends.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from need_b200 import abi
from need_b200 import need_kernels as nk
from need_b200 import workloads

pytestmark = pytest.mark.gpu

ERR_LOOKBACK = 1


@pytest.mark.parametrize("trial", range(3))
def test_lookback_wait_gives_up_and_reports(cuda, trial):
    lib = abi.load()
    B, T, C = 2, 2048, 512
    w = workloads.gated_inputs(B, T, C, z_mean=4.0, dtype=torch.bfloat16, device=cuda, seed=31 + trial,
                               resets="lognormal", seg_lo=16, seg_hi=1024)
    nbytes = lib.need_scan_workspace_size(abi.FORM_GATED, abi.BF16, abi.BF16, 0, B, 1, T, C)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    out = torch.full_like(w.x, float("nan"))
    a = abi.NeedScanArgs()
    nk._fill_common(a, abi.FORM_GATED, torch.bfloat16, B, 1, T, C, out)
    for k, t in enumerate((w.z, w.g, w.x)):
        a.in_[k] = abi.NeedView(t.data_ptr(), t.stride(0), 0, t.stride(1))
    a.seg_start = w.seg.data_ptr()
    a.seg_stride_b, a.seg_stride_t = w.seg.stride()
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    lib.need_test_set_lookback_polls(4)
    try:
        abi.check("need_gated_scan", lib.need_gated_scan(ctypes.byref(a), stream))
        torch.cuda.synchronize()  # the launch completes
    finally:
        lib.need_test_set_lookback_polls(0)
    err = ctypes.c_uint32(0)
    abi.check("need_workspace_error", lib.need_workspace_error(ws.data_ptr(), ctypes.byref(err), stream))
    assert err.value & ERR_LOOKBACK, f"error word {err.value:#x}: no look-back wait gave up"
    assert torch.isfinite(out.float()).all(), "a tile stopped before writing its outputs"

    # the context is still usable: the same scan with a good workspace is right
    got = nk.gated_scan(w.x, w.z, w.g, seg_start=w.seg)
    torch.cuda.synchronize()
    assert nk.workspace_error() == 0
    want, _ = oracle.gated_scan(*(t.float().cpu().numpy() for t in (w.x, w.z, w.g)), w.seg.cpu().numpy(),
                                dtype="bf16")
    g = got.float().cpu().numpy()
    assert np.abs(g - want).max() <= 2e-2 * np.abs(want).max()
    assert np.mean(g == want) >= 0.99
