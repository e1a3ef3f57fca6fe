"""The SSD block's prologue u = silu(causal depthwise conv_K(u)) in one kernel
(need_core.py:1620-1622), against the reference's own formulation on the CPU:
nn.Conv1d-style conv1d with padding K-1 trimmed to T, rounded to the input
dtype, then SiLU, rounded again.  Tolerance: bf16 2e-2 / f16 5e-3 relative,
and at least 99% of outputs bit-identical.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from need_b200 import need_kernels as nk

pytestmark = pytest.mark.gpu
TOL = {torch.bfloat16: 2e-2, torch.float16: 5e-3}


def reference(u, w, b, seg=None):
    """fp32 conv (the reference's rounding points), per segment when seg is given."""
    B, T, C = u.shape
    K = w.shape[-1]

    def conv(x):  # x [T', C] fp32 -> [T', C]
        y = F.conv1d(x.t().unsqueeze(0), w.float().reshape(C, 1, K), None if b is None else b.float(),
                     padding=K - 1, groups=C)[..., :x.shape[0]]
        return y[0].t()

    out = torch.empty(B, T, C)
    for bi in range(B):
        starts = [0] if seg is None else sorted(set([0] + torch.nonzero(seg[bi]).flatten().tolist()))
        ends = starts[1:] + [T]
        for s, e in zip(starts, ends):
            yc = conv(u[bi, s:e].float()).to(u.dtype).float()
            out[bi, s:e] = F.silu(yc)
    return out.to(u.dtype)


def compare(got, want, dtype):
    g, wv = got.float().cpu(), want.float()
    assert (g - wv).abs().max() <= TOL[dtype] * wv.abs().max(), float((g - wv).abs().max())
    assert torch.mean((g == wv).float()) >= 0.99


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("K", [1, 2, 3, 4])
def test_conv_silu_matches_reference(cuda, dtype, K):
    gen = torch.Generator().manual_seed(K)
    u = torch.randn(2, 203, 96, generator=gen).to(dtype)
    w = (torch.randn(96, 1, K, generator=gen) * 0.5).to(dtype)
    b = (torch.randn(96, generator=gen) * 0.1).to(dtype)
    got = nk.ssd_conv_silu(u.to(cuda), w.to(cuda), b.to(cuda))
    compare(got, reference(u, w, b), dtype)


def test_conv_silu_strided_chunk_no_bias(cuda):
    """u as one chunk of an in-projection output (stride 5C along T), no bias."""
    gen = torch.Generator().manual_seed(9)
    C = 832
    proj = torch.randn(2, 300, 5 * C, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 1, 3, generator=gen) * 0.5).to(torch.bfloat16)
    u = proj.to(cuda)[..., :C]
    assert u.stride(1) == 5 * C
    got = nk.ssd_conv_silu(u, w.to(cuda))
    compare(got, reference(proj[..., :C], w, None), torch.bfloat16)


def test_conv_silu_with_resets(cuda):
    gen = torch.Generator().manual_seed(3)
    B, T, C = 2, 500, 64
    u = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 1, 3, generator=gen) * 0.5).to(torch.bfloat16)
    b = (torch.randn(C, generator=gen) * 0.1).to(torch.bfloat16)
    seg = torch.zeros(B, T, dtype=torch.uint8)
    for t in (1, 31, 32, 33, 64, 95, 96, 200, 201, 499):  # around the 32-token thread chunks
        seg[0, t] = 1
    seg[1, ::7] = 1
    got = nk.ssd_conv_silu(u.to(cuda), w.to(cuda), b.to(cuda), seg_start=seg.to(cuda))
    compare(got, reference(u, w, b, seg), torch.bfloat16)


def test_conv_silu_and_the_fold_against_the_reference_fixture(cuda):
    """Against the activated u captured from the reference's own
    StructuredDualRetention.forward (tests/golden/ssd_prologue_bf16.npz, which
    the oracle reproduces bit for bit): the prologue kernel, and the conv that
    ssd_conv_scan folds into the scan (bit-identical to the prologue kernel, so
    its scan of the fixture's u_act equals ssd_scan of the kernel's)."""
    import os
    import sys
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, here)
    import cases  # noqa: E402
    inp = cases.make_inputs("ssd_prologue_bf16")
    want = torch.from_numpy(np.load(os.path.join(here, "ssd_prologue_bf16.npz"))["u_act"])
    u = torch.from_numpy(inp["u"]).to(torch.bfloat16).to(cuda)
    n, t, c = u.shape
    w = torch.from_numpy(inp["conv_w"]).to(torch.bfloat16).view(c, 1, -1).to(cuda)
    b = torch.from_numpy(inp["conv_b"]).to(torch.bfloat16).to(cuda)
    got = nk.ssd_conv_silu(u, w, b)
    compare(got, want.to(torch.bfloat16), torch.bfloat16)
    gen = torch.Generator(device=cuda).manual_seed(2)
    bg, cg, dt, og = (torch.randn(n, t, c, device=cuda, generator=gen).to(torch.bfloat16) for _ in range(4))
    d = torch.full((c,), 0.1, device=cuda)
    fold = nk.ssd_conv_scan(u, bg, cg, dt, og, d, 0.001, 0.2, w, b)
    assert torch.equal(fold, nk.ssd_scan(got, bg, cg, dt, og, d, 0.001, 0.2))
    # a u_act one unit off moves the state of every later token, so only the tolerance applies here
    via_fixture = nk.ssd_scan(want.to(torch.bfloat16).to(cuda), bg, cg, dt, og, d, 0.001, 0.2).float()
    assert (fold.float() - via_fixture).abs().max() <= TOL[torch.bfloat16] * via_fixture.abs().max()
