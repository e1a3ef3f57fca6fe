"""The SSD block's out_norm: need_rms_norm (need_kernels.rms_norm on CUDA) and
the scan with the norm after it in one call (need_core.py:1624-1643:
out_norm(ssd_scan(...))), against the oracle: the reference's ssd_scan followed
by the reference's GPU rms_norm arithmetic (need_kernels.py:99-107).

Tolerances as for the scan: fp32 1e-5 relative; 16-bit 2e-2 relative with at
least 99% of outputs bit-identical.  Against the same normalisation applied by
torch ops to this library's own ssd_scan output, the fused kernel differs only
by the order of the fp32 sum of squares: 99.9% of outputs bit-identical.
Repeated calls are bit-identical (the sums are added in a fixed order).
"""
import numpy as np
import pytest
import torch

import cases
import oracle
from need_b200 import need_kernels as nk

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 5e-3}
NAME = {torch.float32: "fp32", torch.bfloat16: "bf16", torch.float16: "fp16"}


def host(t):
    return t.detach().float().cpu().numpy()


def check(got, want, dtype, what=""):
    r = float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))
    assert r <= TOL[dtype], f"{what}: rel err {r}"
    if dtype != torch.float32:
        frac = float(np.mean(got == want))
        assert frac >= 0.99, f"{what}: only {frac:.5f} of outputs equal"


def inputs(B, T, C, dtype, seed, resets=False):
    gen = torch.Generator().manual_seed(seed)
    xs = [torch.randn(B, T, C, generator=gen).to(dtype) for _ in range(5)]  # u, bg, cg, dt, og
    dskip = 0.1 + 0.05 * torch.randn(C, generator=gen)
    w = 1.0 + 0.1 * torch.randn(C, generator=gen)
    seg = None
    if resets:
        seg = (torch.rand(B, T, generator=gen) < 0.02).to(torch.uint8)
        seg[:, 0] = 1
        seg[0, T - 1] = 1
    return xs, dskip, w, seg


def oracle_norm(xs, dskip, w, seg, dtype, eps, h0=None):
    u, bg, cg, dt, og = (x.float().numpy() for x in xs)
    y, hf = oracle.ssd_scan(u, bg, cg, dt, og, dskip.numpy(), 0.001, 0.2,
                            None if seg is None else seg.numpy(),
                            None if h0 is None else h0.numpy(), dtype=NAME[dtype])
    return oracle.rms_norm(y, w.float().numpy(), eps, dtype=NAME[dtype]), hf


def no_device_error():
    assert nk.workspace_error() == 0, "a device-side wait gave up"


@pytest.mark.parametrize("name", ["ssd_norm_fp32", "ssd_norm_bf16"])
def test_matches_reference_fixture(cuda, name):
    inp = cases.make_inputs(name)
    g = np.load(f"{cases.__file__.rsplit('/', 1)[0]}/{name}.npz")
    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16}[cases.CASES[name]["dtype"]]
    args = [torch.from_numpy(inp[k]).to(cuda).to(dtype) for k in ("u", "bg", "cg", "dt", "og")]
    w = torch.from_numpy(inp["norm_w"]).to(cuda)
    got = nk.ssd_scan_rms_norm(*args, torch.from_numpy(inp["dskip"]).to(cuda), inp["dt_min"], inp["dt_max"],
                               w, inp["eps"])
    assert got.dtype == dtype and got.shape == args[0].shape
    if dtype == torch.float32:
        check(host(got), g["norm"], dtype, name)  # the reference's own output
    else:
        # the reference's GPU arithmetic on the reference's own scan output
        check(host(got), oracle.rms_norm(g["y"], inp["norm_w"], inp["eps"], dtype="bf16"), dtype, name)
    no_device_error()


@pytest.mark.parametrize("B,T,C,dtype,resets", [
    (2, 333, 832, torch.bfloat16, True),     # NEED's d_model: 7 channel tiles, the last half full
    (1, 64, 128, torch.bfloat16, False),     # one tile
    (3, 200, 96, torch.float16, True),       # one partial tile
    (2, 130, 520, torch.float32, True),      # fp32: 256-channel tiles
    (1, 70, 8192, torch.bfloat16, False),    # 64 channel tiles per token chunk
    (2, 50, 8200, torch.bfloat16, True),     # 65 channel tiles, the last one 8 channels wide
])
def test_matches_oracle(cuda, B, T, C, dtype, resets):
    xs, dskip, w, seg = inputs(B, T, C, dtype, seed=C + T, resets=resets)
    h0 = torch.randn(B, C, generator=torch.Generator().manual_seed(1)) * 0.5
    hf = torch.empty(B, C, device=cuda)
    got = nk.ssd_scan_rms_norm(*[x.to(cuda) for x in xs], dskip.to(cuda), 0.001, 0.2, w.to(cuda), 1e-6,
                               seg_start=None if seg is None else seg.to(cuda), h0=h0.to(cuda), h_final=hf)
    want, want_hf = oracle_norm(xs, dskip, w, seg, dtype, 1e-6, h0=h0)
    check(host(got), want, dtype, f"{B}x{T}x{C}")
    # the fp32 final state: a one-ulp difference in a 16-bit gate moves it by ~2^-11 (fp16)
    hf_tol = {torch.float32: 1e-5, torch.bfloat16: 1e-3, torch.float16: 5e-3}[dtype]
    assert float(np.abs(host(hf) - want_hf).max() / max(np.abs(want_hf).max(), 1e-30)) <= hf_tol
    no_device_error()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_same_as_unfused_on_gpu(cuda, dtype):
    """Fused against ssd_scan followed by the same normalisation as torch ops."""
    xs, dskip, w, seg = inputs(4, 1000, 832, dtype, seed=5, resets=True)
    xs = [x.to(cuda) for x in xs]
    args = (*xs, dskip.to(cuda), 0.001, 0.2)
    seg = seg.to(cuda)
    y = nk.ssd_scan(*args, seg_start=seg)
    want = nk._rms_norm_gpu(y, w.to(cuda), 1e-6)
    got = nk.ssd_scan_rms_norm(*args, w.to(cuda), 1e-6, seg_start=seg)
    g, wv = host(got), host(want)
    assert float(np.mean(g == wv)) >= 0.999
    assert float(np.abs(g - wv).max() / np.abs(wv).max()) <= TOL[dtype]
    no_device_error()


def test_weight_in_model_dtype_and_projection_chunks(cuda):
    """A bf16 model: bf16 norm weight, and the five gates as chunks of one
    in-projection output (stride 5*D along T), as need_core.py:1619 makes them."""
    gen = torch.Generator().manual_seed(4)
    B, T, D = 2, 257, 832
    proj = torch.randn(B, T, 5 * D, generator=gen).to(torch.bfloat16)
    dskip = torch.full((D,), 0.1)
    w = (1.0 + 0.1 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    u, bg, cg, dt, og = proj.to(cuda).chunk(5, dim=-1)
    assert u.stride(1) == 5 * D
    got = nk.ssd_scan_rms_norm(u, bg, cg, dt, og, dskip.to(cuda), 0.001, 0.2, w.to(cuda), 1e-6)
    xs = [c.contiguous() for c in proj.chunk(5, dim=-1)]
    want, _ = oracle_norm(xs, dskip, w, None, torch.bfloat16, 1e-6)
    check(host(got), want, torch.bfloat16, "projection chunks")
    no_device_error()


@pytest.mark.parametrize("C", [100, 36])
def test_widths_outside_the_fused_kernel(cuda, C):
    """D not a multiple of 8: the scan kernel and the normalisation as torch
    ops, same arithmetic."""
    xs, dskip, w, _ = inputs(1, 40, C, torch.bfloat16, seed=C)
    got = nk.ssd_scan_rms_norm(*[x.to(cuda) for x in xs], dskip.to(cuda), 0.001, 0.2, w.to(cuda), 1e-5)
    want, _ = oracle_norm(xs, dskip, w, None, torch.bfloat16, 1e-5)
    check(host(got), want, torch.bfloat16, f"C={C}")


def test_bad_weight_size(cuda):
    xs, dskip, w, _ = inputs(1, 8, 64, torch.bfloat16, seed=0)
    with pytest.raises(ValueError):
        nk.ssd_scan_rms_norm(*[x.to(cuda) for x in xs], dskip.to(cuda), 0.001, 0.2, w[:32].to(cuda))


def test_repeat_calls_identical_and_workspace_reuse(cuda):
    """Back-to-back calls on one workspace, with other shapes and forms in
    between, give identical results."""
    xs, dskip, w, seg = inputs(2, 700, 832, torch.bfloat16, seed=8, resets=True)
    args = ([x.to(cuda) for x in xs], dskip.to(cuda), w.to(cuda), seg.to(cuda))
    a = nk.ssd_scan_rms_norm(*args[0], args[1], 0.001, 0.2, args[2], 1e-6, seg_start=args[3])
    xs2, d2, w2, _ = inputs(3, 129, 96, torch.bfloat16, seed=9)
    nk.ssd_scan_rms_norm(*[x.to(cuda) for x in xs2], d2.to(cuda), 0.001, 0.2, w2.to(cuda))
    # other scans in between leave their records in the shared workspace
    g = torch.Generator().manual_seed(3)
    z, gg, x = (torch.randn(4, 1500, 1024, generator=g).to(torch.bfloat16).to(cuda) for _ in range(3))
    nk.gated_scan(z, gg, x)
    xs3, d3, w3, _ = inputs(1, 90, 520, torch.float32, seed=10)
    nk.ssd_scan_rms_norm(*[x.to(cuda) for x in xs3], d3.to(cuda), 0.001, 0.2, w3.to(cuda))
    b = nk.ssd_scan_rms_norm(*args[0], args[1], 0.001, 0.2, args[2], 1e-6, seg_start=args[3])
    assert torch.equal(a, b)
    no_device_error()


@pytest.mark.parametrize("dtype,wdtype,rows,C", [
    (torch.bfloat16, torch.float32, 3000, 832),
    (torch.bfloat16, torch.bfloat16, 17, 8192),
    (torch.float16, torch.float32, 100, 96),
    (torch.float32, torch.float32, 50, 520),
])
def test_rms_norm_kernel_matches_oracle(cuda, dtype, wdtype, rows, C):
    """need_kernels.rms_norm on CUDA runs need_rms_norm: the reference's GPU
    arithmetic, against the oracle; repeated calls are identical."""
    gen = torch.Generator().manual_seed(rows + C)
    x = (torch.randn(2, rows, C, generator=gen) * 3.0).to(dtype)
    w = (1.0 + 0.1 * torch.randn(C, generator=gen)).to(wdtype)
    got = nk.rms_norm(x.to(cuda), w.to(cuda), 1e-6)
    assert got.dtype == dtype and got.shape == x.shape
    want = oracle.rms_norm(x.float().numpy(), w.float().numpy(), 1e-6, dtype=NAME[dtype])
    g = host(got)
    assert float(np.abs(g - want).max() / np.abs(want).max()) <= TOL[dtype]
    if dtype != torch.float32:  # fp32 keeps rsqrt's last-ulp difference from the oracle's 1/sqrt
        assert float(np.mean(g == want)) >= 0.999
    assert torch.equal(got, nk.rms_norm(x.to(cuda), w.to(cuda), 1e-6))


def test_rms_norm_keeps_the_torch_path_elsewhere(cuda):
    """Under grad, or for shapes the reference's kernel does not take, the
    reference's torch expression (need_kernels.py:276)."""
    x = torch.randn(4, 8, 64, device=cuda, requires_grad=True)
    w = torch.ones(64, device=cuda)
    y = nk.rms_norm(x, w)
    y.sum().backward()
    assert x.grad is not None
    xc = torch.randn(3, 10, 12).to(torch.bfloat16)  # CPU
    ref = xc * torch.rsqrt(xc.float().pow(2).mean(dim=-1, keepdim=True) + 1e-6).to(xc.dtype) * torch.ones(12)
    assert torch.equal(nk.rms_norm(xc, torch.ones(12)), ref)
