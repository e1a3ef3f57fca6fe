"""The SSD block's conv + SiLU folded into the SSD scan (need_ssd_conv_scan,
need_core.py:1620-1629) against the two-kernel sequence it replaces,
ssd_conv_silu then ssd_scan (each pinned to the reference on its own): the
folded kernel computes the same operations in the same order, so every output
must be bit-identical -- across tap counts, both 16-bit dtypes, ragged T,
packed-segment resets on both sides of the tiles' warp and tile edges, an
in-projection chunk as the input, initial / final state and the RMSNorm
epilogue."""
import pytest
import torch

from need_b200 import need_kernels as nk

pytestmark = pytest.mark.gpu


def inputs(B, T, C, dtype, K, seed, device, chunked=False):
    g = torch.Generator(device=device).manual_seed(seed)
    if chunked:  # the five chunks of one in-projection output, stride 5C along T
        proj = torch.randn(B, T, 5 * C, device=device, generator=g).to(dtype)
        u, bg, cg, dt, og = proj.chunk(5, dim=-1)
    else:
        u, bg, cg, dt, og = (torch.randn(B, T, C, device=device, generator=g).to(dtype) for _ in range(5))
    w = (torch.randn(C, 1, K, device=device, generator=g) * 0.5).to(dtype)
    b = (torch.randn(C, device=device, generator=g) * 0.1).to(dtype)
    d = torch.randn(C, device=device, generator=g) * 0.1
    return u, bg, cg, dt, og, d, w, b


def two_kernels(u, bg, cg, dt, og, d, w, b, seg=None, h0=None, h_final=None):
    ua = nk.ssd_conv_silu(u, w, b, seg_start=seg)
    return nk.ssd_scan(ua, bg, cg, dt, og, d, 0.001, 0.2, seg_start=seg, h0=h0, h_final=h_final)


def resets(B, T, device):
    seg = torch.zeros(B, T, dtype=torch.uint8, device=device)
    # around the 16-row warp edges and the 64-token tile edges
    for t in (1, 2, 15, 16, 17, 18, 47, 48, 63, 64, 65, 66, 127, 128, 130, 191):
        if t < T:
            seg[0, t] = 1
    seg[-1, ::5] = 1
    return seg


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("K", [1, 2, 3, 4])
def test_bit_identical_to_prologue_then_scan(cuda, dtype, K):
    args = inputs(2, 203, 832, dtype, K, seed=K, device=cuda)
    want = two_kernels(*args)
    got = nk.ssd_conv_scan(*args[:6], 0.001, 0.2, args[6], args[7])
    assert torch.equal(got, want)


@pytest.mark.parametrize("K", [2, 3, 4])
def test_bit_identical_with_resets(cuda, K):
    args = inputs(3, 300, 128, torch.bfloat16, K, seed=10 + K, device=cuda)
    seg = resets(3, 300, cuda)
    want = two_kernels(*args, seg=seg)
    got = nk.ssd_conv_scan(*args[:6], 0.001, 0.2, args[6], args[7], seg_start=seg)
    assert torch.equal(got, want)


def test_model_shape_chunked_input_no_bias(cuda):
    """NEED's 350M shape (B=8, T=2048, d_model=832, K=3) with the five inputs as
    chunks of one in-projection output, and a conv without bias."""
    u, bg, cg, dt, og, d, w, _ = inputs(8, 2048, 832, torch.bfloat16, 3, seed=5, device=cuda, chunked=True)
    assert u.stride(1) == 5 * 832
    want = two_kernels(u, bg, cg, dt, og, d, w, None)
    got = nk.ssd_conv_scan(u, bg, cg, dt, og, d, 0.001, 0.2, w, None)
    assert torch.equal(got, want)
    assert nk.workspace_error() == 0


def test_initial_and_final_state(cuda):
    args = inputs(2, 500, 256, torch.bfloat16, 3, seed=21, device=cuda)
    h0 = torch.randn(2, 256, device=cuda)
    hf_want, hf_got = torch.empty(2, 256, device=cuda), torch.empty(2, 256, device=cuda)
    want = two_kernels(*args, h0=h0, h_final=hf_want)
    got = nk.ssd_conv_scan(*args[:6], 0.001, 0.2, args[6], args[7], h0=h0, h_final=hf_got)
    assert torch.equal(got, want)
    assert torch.equal(hf_got, hf_want)


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
def test_with_out_norm(cuda, wdtype):
    args = inputs(4, 1000, 832, torch.bfloat16, 3, seed=33, device=cuda)
    nw = (1.0 + 0.1 * torch.randn(832, device=cuda)).to(wdtype)
    seg = resets(4, 1000, cuda)
    ua = nk.ssd_conv_silu(args[0], args[6], args[7], seg_start=seg)
    want = nk.ssd_scan_rms_norm(ua, *args[1:6], 0.001, 0.2, nw, 1e-6, seg_start=seg)
    got = nk.ssd_conv_scan(*args[:6], 0.001, 0.2, args[6], args[7], norm_weight=nw, eps=1e-6, seg_start=seg)
    assert torch.equal(got, want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_partial_channel_block(cuda, dtype):
    """C=200: three full 64-channel tiles and one of 8 channels, with resets."""
    args = inputs(2, 333, 200, dtype, 3, seed=40, device=cuda)
    seg = resets(2, 333, cuda)
    want = two_kernels(*args, seg=seg)
    got = nk.ssd_conv_scan(*args[:6], 0.001, 0.2, args[6], args[7], seg_start=seg)
    assert torch.equal(got, want)


def test_single_token_and_short_sequences(cuda):
    for T in (1, 2, 3, 17, 64, 65):
        args = inputs(2, T, 64, torch.bfloat16, 3, seed=T, device=cuda)
        assert torch.equal(nk.ssd_conv_scan(*args[:6], 0.001, 0.2, args[6], args[7]), two_kernels(*args)), T
